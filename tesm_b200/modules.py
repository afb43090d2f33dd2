"""Mirror of the reference module API, backed by the sm_100a kernels.

The classes keep the reference's constructor signatures, parameter/buffer names
and the order in which construction consumes the torch RNG, so that
``torch.manual_seed(s)`` followed by construction yields the same state_dict as
the reference (WANGLILIN360/tesm) and checkpoints load with ``strict=True``.

References (paths relative to the reference project):
  BitLinear            tesm_ssm/modules/tesm.py:124-290
  TESM_SISO            tesm_ssm/modules/tesm.py:456-1400
  TESMMIMO_Optimized   tesm_ssm/modules/tesm_mimo.py:76-1062
  RMSNorm, Block       tesm_ssm/modules/block.py:7-50

The only accepted ``kernel_backend`` for a forward pass is ``"b200"``; any other
value, training mode, grad mode or a CPU tensor raises the reference-style
``RuntimeError("kernel_backend='...' specified but ... not available ...")``
(pattern of tesm.py:279-285).  There is no CPU fallback.
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn

from . import layers

B200 = "b200"


class BitLinear(nn.Module):
    """Ternary-weight linear layer (tesm.py:124-290), int8 x int2 on sm_100a.

    Forward: per-tensor absmean ternary weight (tesm.py:211-215), per-token int8
    absmax activation (tesm.py:206-209), exact int32 accumulation, output scaled by
    the two dequantisation factors, in the input dtype.
    """

    def __init__(self, in_features, out_features, bias=False, bit_eps=1e-5, bit_threshold=0.5,
                 kernel_backend=B200, kernel_mode="fast", device=None, dtype=None):
        super().__init__()
        factory_kwargs = {"device": device, "dtype": dtype}
        self.in_features = in_features
        self.out_features = out_features
        self.bit_eps = bit_eps
        self.bit_threshold = bit_threshold
        self.kernel_backend = str(kernel_backend)
        self.kernel_mode = "precise" if str(kernel_mode) == "precise" else "fast"
        self.weight = nn.Parameter(torch.empty(out_features, in_features, **factory_kwargs))
        if bias:
            self.bias = nn.Parameter(torch.zeros(out_features, **factory_kwargs))
        else:
            self.bias = None
        self._b200 = None  # device-side packed weight cache (layers.PackedWeight)
        self.reset_parameters()

    def reset_parameters(self):
        nn.init.kaiming_uniform_(self.weight, a=math.sqrt(5))
        if self.bias is not None:
            bound = 1 / math.sqrt(self.in_features)
            nn.init.uniform_(self.bias, -bound, bound)

    def forward(self, x):
        layers.require_b200(self, x, "BitLinear")
        return layers.bitlinear_forward(self, x)


class TernaryQuantumTunneling(nn.Module):
    """Parameter/buffer mirror of tesm.py:294-445 (eval-time ternary tunneling rule)."""

    def __init__(self, threshold=0.1, tunneling_strength=0.1, num_tunnel_paths=4, min_tunnel_prob=0.05,
                 max_tunnel_prob=0.5, device=None, dtype=None):
        super().__init__()
        self.threshold = threshold
        self.tunneling_strength = tunneling_strength
        self.num_tunnel_paths = num_tunnel_paths
        self.min_tunnel_prob = min_tunnel_prob
        self.max_tunnel_prob = max_tunnel_prob
        self.tunnel_scale = nn.Parameter(torch.ones(1, device=device, dtype=torch.float32))
        self.register_buffer("tunnel_step", torch.tensor(0))
        self.register_buffer("tunnel_to_positive", torch.tensor(0))
        self.register_buffer("tunnel_to_negative", torch.tensor(0))
        self.register_buffer("tunnel_to_zero", torch.tensor(0))
        self.register_buffer("total_boundary", torch.tensor(0))


class TESM_SISO(nn.Module):
    """Single-head TESM mixer (tesm.py:456-1400) on the b200 kernels."""

    def __init__(self, d_model, d_state=256, expand=2, ent_rank=64, entanglement_scale=0.2,
                 entanglement_threshold=0.1, max_seq_len=2048, dropout=0.0, bit_eps=1e-5, bit_threshold=0.5,
                 layer_idx=None, device=None, dtype=None, annealing_enabled=True, T_start=10.0, T_end=0.1,
                 annealing_steps=1000, annealing_schedule="cosine", quantum_tunneling_enabled=False,
                 tunneling_strength=0.1, num_tunnel_paths=4, energy_landscape="entropy",
                 tunneling_schedule="adaptive", **kwargs):
        super().__init__()
        self.d_model = d_model
        self.d_state = d_state
        self.expand = expand
        if d_state <= 0:
            raise ValueError(f"d_state must be positive, got {d_state}")
        if d_model <= 0:
            raise ValueError(f"d_model must be positive, got {d_model}")
        if ent_rank <= 0:
            raise ValueError(f"ent_rank must be positive, got {ent_rank}")
        if max_seq_len <= 0:
            raise ValueError(f"max_seq_len must be positive, got {max_seq_len}")
        self.ent_rank = ent_rank
        self.entanglement_scale = entanglement_scale
        self.entanglement_threshold = entanglement_threshold
        self.entanglement_init = kwargs.get("entanglement_init", 0.3)
        self.entanglement_window = int(kwargs.get("entanglement_window", 0) or 0)
        self.entanglement_block_size = int(kwargs.get("entanglement_block_size", 256) or 256)
        self.state_scan_chunk_size = int(kwargs.get("state_scan_chunk_size", 16) or 16)
        self.use_triton_kernels = bool(kwargs.get("use_triton_kernels", True))
        self.kernel_backend = str(kwargs.get("kernel_backend", B200))
        self.kernel_mode = "precise" if str(kwargs.get("kernel_mode", "fast")) == "precise" else "fast"
        self.max_seq_len = max_seq_len
        self.layer_idx = layer_idx
        self.annealing_enabled = annealing_enabled
        self.T_start = T_start
        self.T_end = T_end
        self.annealing_steps = annealing_steps
        self.annealing_schedule = annealing_schedule
        self.register_buffer("annealing_step", torch.tensor(0))
        self.quantum_tunneling_enabled = quantum_tunneling_enabled
        if quantum_tunneling_enabled:
            self.quantum_tunneler = TernaryQuantumTunneling(threshold=entanglement_threshold,
                                                            tunneling_strength=tunneling_strength,
                                                            num_tunnel_paths=num_tunnel_paths, device=device,
                                                            dtype=dtype)
        else:
            self.quantum_tunneler = None
        bl = dict(bias=False, bit_eps=bit_eps, bit_threshold=bit_threshold, kernel_backend=self.kernel_backend,
                  kernel_mode=self.kernel_mode, device=device, dtype=dtype)
        total_proj = (2 * d_model) + (3 * d_state) + (2 * ent_rank)
        self.in_proj = BitLinear(d_model, total_proj, **bl)
        self.state_proj = BitLinear(d_state, d_model, **bl)
        self.ent_proj = BitLinear(d_state, d_model, **bl)
        self.out_proj = BitLinear(d_model, d_model, **bl)
        self.dropout = nn.Dropout(dropout)
        decay_init = float(kwargs.get("decay_init_bias", 3.0))
        self.decay_bias = nn.Parameter(torch.full((d_state,), decay_init, device=device, dtype=torch.float32))
        if self.entanglement_window > 0:
            self.register_parameter("entanglement", None)
            self.local_entanglement_bias = nn.Parameter(
                torch.randn(self.entanglement_window, device=device, dtype=torch.float32) * self.entanglement_init)
            self.register_parameter("global_entanglement_bias", None)
        else:
            self.register_parameter("local_entanglement_bias", None)
            self.global_rel_pos_scale = nn.Parameter(torch.ones(1, device=device, dtype=torch.float32))
            self.global_rel_pos_bias = nn.Parameter(torch.zeros(1, device=device, dtype=torch.float32))
            self.global_rel_pos_dim = int(kwargs.get("global_rel_pos_dim", 64))
            self.global_rel_pos_embed = nn.Parameter(
                torch.randn(self.global_rel_pos_dim, device=device, dtype=torch.float32) * 0.02)
            self.register_parameter("global_entanglement_bias", None)
            self.register_parameter("entanglement", None)
        self.rope_base = float(kwargs.get("rope_base", 10000.0))
        self.cross_layer_q_proj = BitLinear(d_state, ent_rank, **bl)
        self.last_entanglement_map = None
        self.last_entanglement_stats = None
        self._last_cross_layer_state = None
        self._last_scan_state_f64 = None

    def get_temperature(self):
        """Eval-mode temperature (tesm.py:587-595): T_end."""
        return self.T_end

    def allocate_inference_cache(self, batch_size, max_seqlen, dtype=None, **kwargs):
        """Decode cache with the reference's dict keys (tesm.py:620-670)."""
        return layers.siso_alloc_cache(self, batch_size, max_seqlen, dtype=dtype, **kwargs)

    def forward(self, u, inference_params=None, cross_layer_state=None, prev_state=None, **kwargs):
        layers.require_b200(self, u, "TESM_SISO")
        batch, seqlen, _ = u.shape
        if seqlen > self.max_seq_len:
            raise ValueError(f"Sequence length {seqlen} exceeds max_seq_len {self.max_seq_len}")
        if seqlen == 0:
            return u, None
        if inference_params is not None and seqlen == 1:
            layer_cache = inference_params.get("state_cache")
            if layer_cache is not None and "state" in layer_cache:
                return layers.siso_decode(self, u, layer_cache, cross_layer_state)
        cache = inference_params.get("state_cache") if inference_params is not None else None
        return layers.siso_prefill(self, u, cross_layer_state, prev_state, cache)


class TESMMIMO_Optimized(TESM_SISO):
    """Multi-head TESM mixer (tesm_mimo.py:76-1062) on the b200 kernels."""

    def __init__(self, d_model, d_state=256, n_heads=4, mimo_rank=4, expand=2, ent_rank=48, entanglement_window=16,
                 max_seq_len=2048, entanglement_threshold=0.5, dropout=0.0, bit_eps=1e-5, bit_threshold=0.5,
                 kernel_backend=B200, annealing_enabled=True, T_start=10.0, T_end=0.1, annealing_steps=1000,
                 annealing_schedule="cosine", **kwargs):
        kwargs.setdefault("kernel_backend", kernel_backend)
        super().__init__(d_model=d_model, d_state=d_state, expand=expand, ent_rank=ent_rank,
                         entanglement_window=entanglement_window, max_seq_len=max_seq_len,
                         entanglement_threshold=entanglement_threshold, dropout=dropout, bit_eps=bit_eps,
                         bit_threshold=bit_threshold, annealing_enabled=annealing_enabled, T_start=T_start,
                         T_end=T_end, annealing_steps=annealing_steps, annealing_schedule=annealing_schedule,
                         **kwargs)
        self.n_heads = n_heads
        self.mimo_rank = mimo_rank
        self.d_inner = int(expand * d_model)
        self.d_head = self.d_inner // n_heads
        self.d_state_total = d_state * n_heads
        self.kernel_backend = kernel_backend
        device = kwargs.get("device")
        decay_init = float(kwargs.get("decay_init_bias", 3.0))
        self.decay_bias = nn.Parameter(torch.full((n_heads, d_state), decay_init, device=device, dtype=torch.float32))
        if entanglement_window > 0:
            self.local_entanglement_bias = nn.Parameter(
                torch.randn(n_heads, entanglement_window, device=device, dtype=torch.float32) * 0.02)
        else:
            self.register_parameter("local_entanglement_bias", None)
        self.rope_base = float(kwargs.get("rope_base", 10000.0))
        self.mimo_x = nn.Parameter(torch.ones(n_heads, mimo_rank, d_state, device=device, dtype=torch.float32) / mimo_rank)
        self.mimo_z = nn.Parameter(torch.ones(n_heads, mimo_rank, d_state, device=device, dtype=torch.float32))
        self.mimo_o = nn.Parameter(torch.ones(n_heads, mimo_rank, d_state, device=device, dtype=torch.float32) / mimo_rank)
        bl = dict(bias=False, bit_eps=bit_eps, bit_threshold=bit_threshold, kernel_backend=kernel_backend,
                  device=device, dtype=kwargs.get("dtype"))
        d_in = (2 * d_model) + (3 * d_state * n_heads) + (2 * ent_rank * n_heads)
        self.in_proj = BitLinear(d_model, d_in, **bl)
        self.state_proj = BitLinear(self.d_state_total, d_model, **bl)
        self.ent_proj = BitLinear(self.d_state_total, d_model, **bl)

    def allocate_inference_cache(self, batch_size, max_seqlen, dtype=None, **kwargs):
        """Decode cache with the reference's dict keys (tesm_mimo.py:689-731)."""
        return layers.mimo_alloc_cache(self, batch_size, max_seqlen, dtype=dtype, **kwargs)

    def forward(self, u, inference_params=None, cross_layer_state=None, prev_state=None, **kwargs):
        layers.require_b200(self, u, "TESMMIMO_Optimized")
        batch, seqlen, _ = u.shape
        if inference_params is not None and seqlen == 1:
            layer_cache = inference_params.get("state_cache")
            if layer_cache is not None and "state" in layer_cache:
                return layers.mimo_decode(self, u, layer_cache, cross_layer_state)
        cache = inference_params.get("state_cache") if inference_params is not None else None
        return layers.mimo_prefill(self, u, cache)


TESM = TESM_SISO


class RMSNorm(nn.Module):
    """RMSNorm (block.py:7-17)."""

    def __init__(self, dim: int, eps: float = 1e-5):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))

    def forward(self, x):
        return layers.rmsnorm(self, x)


class Block(nn.Module):
    """Pre-norm residual block (block.py:19-50)."""

    def __init__(self, dim, mixer_cls, mlp_cls, norm_cls=nn.LayerNorm, residual_in_fp32=False):
        super().__init__()
        self.residual_in_fp32 = residual_in_fp32
        self.norm = norm_cls(dim)
        self.mixer = mixer_cls(dim)
        self.norm2 = norm_cls(dim)
        self.mlp = mlp_cls(dim)

    def forward(self, hidden_states, residual=None, inference_params=None, prev_state=None, **mixer_kwargs):
        return layers.block_forward(self, hidden_states, residual, inference_params, prev_state, **mixer_kwargs)

    def allocate_inference_cache(self, batch_size, max_seqlen, dtype=None, **kwargs):
        if hasattr(self.mixer, "allocate_inference_cache"):
            return self.mixer.allocate_inference_cache(batch_size, max_seqlen, dtype=dtype, **kwargs)
        return None
