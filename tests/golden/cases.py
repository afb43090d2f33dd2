"""Case table shared by the golden generator and the parity tests.

Each entry names a reference module configuration (keyword arguments exactly as
the reference constructors take them), the batch/sequence shape, and which
optional inputs (cross-layer state, initial state, decode steps) the case drives.
Inputs are drawn from ``torch.Generator().manual_seed(seed)``: x uses seed 1,
cross-layer state seed 2, prev_state seed 4, decode step s uses seeds 10+s / 20+s.
"""

BITLINEAR = [
    # name, in/out features, input shape, latent weight std, dtype
    dict(name="f32", K=96, N=80, xshape=(3, 7, 96), wstd=0.02, dtype="float32"),
    dict(name="bf16", K=160, N=72, xshape=(2, 5, 160), wstd=0.02, dtype="bfloat16"),
    dict(name="odd", K=37, N=19, xshape=(4, 37), wstd=1.0, dtype="float32"),
]

_small = dict(d_model=64, d_state=32, ent_rank=16, entanglement_window=8, max_seq_len=64)

SISO = [
    # d_model 256, d_state 64, window 16, batch 2 x 256, fp32
    dict(name="cfg1", B=2, L=256, kw=dict(d_model=256, d_state=64, entanglement_window=16, max_seq_len=256)),
    dict(name="cross_prev", B=2, L=40, cross=True, prev=True, kw=dict(_small)),
    dict(name="decode", B=3, L=20, cross=True, decode=12, kw=dict(_small)),
    dict(name="short_decode", B=2, L=5, decode=6, kw=dict(_small)),
    dict(name="global", B=2, L=48, kw=dict(d_model=64, d_state=32, ent_rank=16, entanglement_window=0, max_seq_len=64)),
    dict(name="win_gt_len", B=2, L=6, kw=dict(_small)),
]

MIMO = [
    dict(name="small", B=2, L=24, kw=dict(d_model=64, d_state=16, n_heads=4, ent_rank=8, entanglement_window=8,
                                         max_seq_len=64)),
    dict(name="decode", B=2, L=12, cross=True, decode=10,
         kw=dict(d_model=64, d_state=16, n_heads=4, ent_rank=8, entanglement_window=8, max_seq_len=64,
                 entanglement_threshold=0.3)),
    dict(name="short", B=1, L=5, kw=dict(d_model=32, d_state=16, n_heads=2, ent_rank=8, entanglement_window=8,
                                        max_seq_len=32)),
    dict(name="global", B=2, L=20, kw=dict(d_model=64, d_state=16, n_heads=4, ent_rank=8, entanglement_window=0,
                                          max_seq_len=64)),
]

_tiny = dict(n_layer=2, d_model=64, d_state=32, ent_rank=16, d_intermediate=96, vocab_size=128,
             max_seq_len=64, entanglement_window=8)

MODEL = [
    dict(name="tiny", B=2, L=12, decode=5, cfg=dict(_tiny)),
    dict(name="tiny_mimo", B=2, L=10, decode=3, cfg=dict(_tiny, use_mimo=True, n_heads=2, d_state=16, ent_rank=8)),
]
