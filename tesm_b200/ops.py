"""Torch-tensor wrappers over the C ABI (device memory, streams and shapes only).

Every function here launches kernels from libtesm_b200.so on the current torch
stream; none computes anything with torch ops.  Tensors must live on the CUDA
device; ownership stays with torch.
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass
from typing import Optional

import torch

from . import _lib

F32, BF16 = 0, 1
LAYOUT_ROWMAJOR, LAYOUT_GEMV = 0, 1
GEMV_MAX_M = 64

_DT = {torch.float32: F32, torch.bfloat16: BF16}


def dtype_code(dt: torch.dtype) -> int:
    try:
        return _DT[dt]
    except KeyError:
        raise _lib.TesmError(f"tesm_b200: unsupported dtype {dt} (float32 or bfloat16)") from None


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _ptr(t: Optional[torch.Tensor]):
    return None if t is None else t.data_ptr()


def round_up(x: int, m: int) -> int:
    return (x + m - 1) // m * m


@dataclass
class PackedWeight:
    """Device-resident ternary weight of one BitLinear.

    packed: (N, Kp/4) uint8 in the reference INT2 byte format, Kp = K rounded up to 256
    tern:   (N, Kp) int8 ternary values for the tensor-core path (None until needed)
    scale:  (1,) or (N,) float32 quantisation scale 1/mean|W|
    deq:    (1,) or (N,) float32 dequantisation factor fl(1/scale)
    """
    packed: torch.Tensor
    tern: Optional[torch.Tensor]
    scale: torch.Tensor
    deq: torch.Tensor
    N: int
    K: int
    per_row: bool


def weight_scale(w: torch.Tensor, eps: float, per_row: bool = False, scale_out=None, deq_out=None):
    N, K = w.shape
    n = N if per_row else 1
    scale = scale_out if scale_out is not None else torch.empty(n, device=w.device, dtype=torch.float32)
    deq = deq_out if deq_out is not None else torch.empty(n, device=w.device, dtype=torch.float32)
    work = torch.empty(N, device=w.device, dtype=torch.float64)
    _lib.call("tesm_b200_weight_scale", w.data_ptr(), dtype_code(w.dtype), N, K, w.stride(0), int(per_row),
              float(eps), scale.data_ptr(), deq.data_ptr(), work.data_ptr(), _stream())
    return scale, deq


def pack_weight(w: torch.Tensor, eps: float = 1e-5, per_row: bool = False, with_tern: bool = True,
                scale: Optional[torch.Tensor] = None) -> PackedWeight:
    """Ternarise and pack a (N, K) weight; ``scale`` overrides the computed 1/mean|W|."""
    assert w.is_cuda and w.dim() == 2 and w.stride(1) == 1
    N, K = w.shape
    Kp = round_up(K, 256)
    if scale is None:
        scale, deq = weight_scale(w, eps, per_row)
    else:
        scale = scale.to(device=w.device, dtype=torch.float32).reshape(-1).contiguous()
        deq = torch.reciprocal(scale)  # not used on the parity path
    packed = torch.empty(N, Kp // 4, device=w.device, dtype=torch.uint8)
    tern = torch.empty(N, Kp, device=w.device, dtype=torch.int8) if with_tern else None
    _lib.call("tesm_b200_pack_ternary", w.data_ptr(), dtype_code(w.dtype), N, K, w.stride(0), int(per_row),
              scale.data_ptr(), packed.data_ptr(), packed.stride(0), _ptr(tern), Kp if tern is not None else 0,
              _stream())
    return PackedWeight(packed, tern, scale, deq, N, K, per_row)


def packed_from_int2(packed: torch.Tensor, weight_scale, K: int, device) -> PackedWeight:
    """PackedWeight from an exported INT2 weight (pack_int2_to_uint8 bytes, (N, ceil(K/4)) uint8,
    and its weight_scale = 1 / mean|W|; int2_quantization.py:21-60): the bytes are kept as they
    are (rows padded with code 1 up to K rounded to 256) and the int8 ternary operand of the
    tensor-core GEMM is unpacked from them on the device."""
    N, kb = packed.shape
    if packed.dtype != torch.uint8 or kb != (K + 3) // 4:
        raise ValueError(f"packed INT2 weight must be uint8 (N, ceil(K/4)) = (N, {(K + 3) // 4}), got "
                         f"{tuple(packed.shape)} {packed.dtype}")
    Kp = round_up(K, 256)
    dev = torch.device(device)
    buf = torch.full((N, Kp // 4), 0x55, device=dev, dtype=torch.uint8)
    buf[:, :kb] = packed.to(dev)
    scale = torch.as_tensor(weight_scale, dtype=torch.float32).reshape(1).to(dev)
    deq = torch.reciprocal(scale)
    tern = torch.empty(N, Kp, device=dev, dtype=torch.int8)
    _lib.call("tesm_b200_unpack_ternary", buf.data_ptr(), buf.stride(0), N, Kp, tern.data_ptr(), tern.stride(0),
              _stream())
    return PackedWeight(buf, tern, scale, deq, N, K, False)


def ensure_tern(pw: PackedWeight, w: torch.Tensor):
    if pw.tern is None:
        Kp = round_up(pw.K, 256)
        tern = torch.empty(pw.N, Kp, device=w.device, dtype=torch.int8)
        scratch = torch.empty_like(pw.packed)
        _lib.call("tesm_b200_pack_ternary", w.data_ptr(), dtype_code(w.dtype), pw.N, pw.K, w.stride(0),
                  int(pw.per_row), pw.scale.data_ptr(), scratch.data_ptr(), scratch.stride(0), tern.data_ptr(), Kp,
                  _stream())
        pw.tern = tern
    return pw.tern


def quant_act(x2d: torch.Tensor, eps: float, layout: int):
    """Per-row int8 codes of a (M, K) activation (row stride may exceed K)."""
    assert x2d.is_cuda and x2d.dim() == 2 and x2d.stride(1) == 1
    M, K = x2d.shape
    ld = round_up(K, 256) if layout == LAYOUT_GEMV else round_up(K, 16)
    codes = torch.empty(M, ld, device=x2d.device, dtype=torch.int8)
    inv = torch.empty(M, device=x2d.device, dtype=torch.float32)
    rowsum = torch.empty(M, device=x2d.device, dtype=torch.int32) if layout == LAYOUT_GEMV else None
    _lib.call("tesm_b200_quant_act", x2d.data_ptr(), dtype_code(x2d.dtype), M, K, x2d.stride(0), float(eps),
              codes.data_ptr(), ld, layout, inv.data_ptr(), _ptr(rowsum), _stream())
    return codes, inv, rowsum


def quant_act_into(x2d: torch.Tensor, eps: float, codes: torch.Tensor, col0: int, inv: torch.Tensor):
    """Row-major int8 codes of x written into columns [col0, col0 + K) of ``codes`` (16-byte
    aligned rows and col0), 1/s into ``inv``."""
    assert x2d.is_cuda and x2d.dim() == 2 and x2d.stride(1) == 1 and col0 % 16 == 0
    M, K = x2d.shape
    _lib.call("tesm_b200_quant_act", x2d.data_ptr(), dtype_code(x2d.dtype), M, K, x2d.stride(0), float(eps),
              codes.data_ptr() + col0, codes.stride(0), LAYOUT_ROWMAJOR, inv.data_ptr(), None, _stream())


def gemv(codes, inv, rowsum, pw: PackedWeight, M: int, out_dtype: torch.dtype, out=None, acc=False):
    dev = codes.device
    out = out if out is not None else torch.empty(M, pw.N, device=dev, dtype=out_dtype)
    accb = torch.empty(M, pw.N, device=dev, dtype=torch.int32) if acc else None
    _lib.call("tesm_b200_gemv_int2", codes.data_ptr(), codes.stride(0), inv.data_ptr(), rowsum.data_ptr(),
              pw.packed.data_ptr(), pw.packed.stride(0), pw.deq.data_ptr(), int(pw.per_row), M, pw.N, pw.K,
              out.data_ptr(), dtype_code(out.dtype), out.stride(0), _ptr(accb), pw.N, _stream())
    return (out, accb) if acc else out


_SPLITK = {}
SPLITK_MAX_M = 1024


SPLITK_COUNTERS = 4096  # int32 tile counters at the start of the scratch (zero between calls)


def splitk_workspace(M: int, N: int, device):
    """int32 split-K scratch shared by the small-M tensor-core GEMMs of a device: tile counters
    (zero-initialised here; every GEMM call leaves them zero again) followed by room for 8
    partial M x N slices.  None for large M, where split-K is never chosen."""
    if M > SPLITK_MAX_M:
        return None
    need = SPLITK_COUNTERS + 8 * round_up(M, 256) * round_up(N, 32)  # slices cover whole tiles
    key = torch.device(device).index
    buf = _SPLITK.get(key)
    if buf is None or buf.numel() < need:
        if buf is not None:
            torch.cuda.current_stream(device).synchronize()  # the old buffer may still be in use
        buf = torch.zeros(max(need, 1 << 20), device=device, dtype=torch.int32)
        _SPLITK[key] = buf
    return buf


def gemm(codes, inv, pw: PackedWeight, M: int, out_dtype: torch.dtype, out=None, acc=False):
    dev = codes.device
    out = out if out is not None else torch.empty(M, pw.N, device=dev, dtype=out_dtype)
    accb = torch.empty(M, pw.N, device=dev, dtype=torch.int32) if acc else None
    ws = splitk_workspace(M, pw.N, dev)
    _lib.call("tesm_b200_gemm_i8", codes.data_ptr(), codes.stride(0), inv.data_ptr(), pw.tern.data_ptr(),
              pw.tern.stride(0), pw.deq.data_ptr(), int(pw.per_row), M, pw.N, pw.K, out.data_ptr(),
              dtype_code(out.dtype), out.stride(0), _ptr(accb), pw.N, _ptr(ws), ws.numel() * 4 if ws is not None else 0,
              _stream())
    return (out, accb) if acc else out


def gemm_bf16(a: torch.Tensor, b: torch.Tensor, out_dtype=torch.bfloat16, out=None):
    """a (M, K) @ b (N, K)^T on the tensor cores (bf16 in, fp32 accumulate)."""
    M, K = a.shape
    N = b.shape[0]
    out = out if out is not None else torch.empty(M, N, device=a.device, dtype=out_dtype)
    _lib.call("tesm_b200_gemm_bf16", a.data_ptr(), a.stride(0), b.data_ptr(), b.stride(0), M, N, K, out.data_ptr(),
              dtype_code(out.dtype), out.stride(0), _stream())
    return out


def gemm_acc(codes, inv, pw: PackedWeight, M: int, acc: torch.Tensor):
    """int32 accumulators only (no scaled output): the partial product of a row-parallel shard."""
    ws = splitk_workspace(M, pw.N, codes.device)
    _lib.call("tesm_b200_gemm_i8", codes.data_ptr(), codes.stride(0), inv.data_ptr(), pw.tern.data_ptr(),
              pw.tern.stride(0), pw.deq.data_ptr(), int(pw.per_row), M, pw.N, pw.K, None, dtype_code(torch.float32),
              pw.N, acc.data_ptr(), acc.stride(0), _ptr(ws), ws.numel() * 4 if ws is not None else 0, _stream())
    return acc


def acc_scale(acc, inv, pw: PackedWeight, out_dtype, out=None):
    """out = acc * inv_scale[row] * deq (the GEMM epilogue's float operations, bit for bit)."""
    M, N = acc.shape
    out = out if out is not None else torch.empty(M, N, device=acc.device, dtype=out_dtype)
    _lib.call("tesm_b200_acc_scale", acc.data_ptr(), M, N, inv.data_ptr(), pw.deq.data_ptr(), int(pw.per_row),
              out.data_ptr(), dtype_code(out.dtype), out.stride(0), _stream())
    return out


def combine_acc(acc1, acc2, inv1, inv2, deq1, deq2, proj, c_local, c_gate, out):
    """The dual-accumulator combine epilogue on summed int32 accumulators (bit for bit)."""
    M, N = out.shape
    _lib.call("tesm_b200_combine_acc", acc1.data_ptr(), acc2.data_ptr(), acc1.stride(0), M, N, inv1.data_ptr(),
              inv2.data_ptr(), deq1.data_ptr(), deq2.data_ptr(), proj.data_ptr(), dtype_code(proj.dtype),
              proj.stride(0), c_local, c_gate, out.data_ptr(), dtype_code(out.dtype), out.stride(0), _stream())
    return out


def row_absmax(x2d: torch.Tensor, out=None):
    M, K = x2d.shape
    out = out if out is not None else torch.empty(M, device=x2d.device, dtype=torch.float32)
    _lib.call("tesm_b200_row_absmax", x2d.data_ptr(), dtype_code(x2d.dtype), M, K, x2d.stride(0), out.data_ptr(),
              _stream())
    return out


def quant_act_amax(x2d: torch.Tensor, eps: float, amax: torch.Tensor) -> "QuantAct":
    """Row-major int8 codes of x with the row maxima given (global across tensor-parallel shards)."""
    M, K = x2d.shape
    ld = round_up(K, 16)
    codes = torch.empty(M, ld, device=x2d.device, dtype=torch.int8)
    inv = torch.empty(M, device=x2d.device, dtype=torch.float32)
    _lib.call("tesm_b200_quant_act_amax", x2d.data_ptr(), dtype_code(x2d.dtype), M, K, x2d.stride(0), float(eps),
              amax.data_ptr(), codes.data_ptr(), ld, LAYOUT_ROWMAJOR, inv.data_ptr(), None, _stream())
    return QuantAct(codes, inv, None, LAYOUT_ROWMAJOR, M)


def pack_shard(w_full: torch.Tensor, eps: float, rows=None, cols=None, per_row: bool = False) -> PackedWeight:
    """Ternary pack of a row or column slice of a weight with the scale of the FULL weight (the
    reference quantises each BitLinear as a whole, tesm.py:211-215)."""
    scale, deq = weight_scale(w_full, eps, per_row)
    w = w_full
    if rows is not None:
        w = w[rows[0]:rows[1]]
        if per_row:
            scale, deq = scale[rows[0]:rows[1]].contiguous(), deq[rows[0]:rows[1]].contiguous()
    if cols is not None:
        w = w[:, cols[0]:cols[1]]
    pw = pack_weight(w, eps, per_row, with_tern=True, scale=scale)
    pw.deq = deq
    return pw


def bitlinear_2d(x2d: torch.Tensor, pw: PackedWeight, eps: float, out_dtype=None, out=None, acc=False,
                 force: Optional[str] = None):
    """Quantise a (M, K) activation and multiply by a packed ternary weight."""
    M = x2d.shape[0]
    out_dtype = out_dtype or x2d.dtype
    path = force or ("gemv" if M <= GEMV_MAX_M else "gemm")
    if path == "gemv":
        codes, inv, rowsum = quant_act(x2d, eps, LAYOUT_GEMV)
        return gemv(codes, inv, rowsum, pw, M, out_dtype, out, acc)
    codes, inv, _ = quant_act(x2d, eps, LAYOUT_ROWMAJOR)
    return gemm(codes, inv, pw, M, out_dtype, out, acc)


# ------------------------------------------------------------------ pre-quantised activations
@dataclass
class QuantAct:
    """int8 activation codes of M rows ready for a BitLinear (layout GEMV or ROWMAJOR)."""
    codes: torch.Tensor
    inv: torch.Tensor
    rowsum: Optional[torch.Tensor]
    layout: int
    M: int


def layout_for(M: int) -> int:
    return LAYOUT_GEMV if M <= GEMV_MAX_M else LAYOUT_ROWMAJOR


def alloc_quant(M: int, K: int, device, layout: Optional[int] = None) -> QuantAct:
    layout = layout_for(M) if layout is None else layout
    ld = round_up(K, 256) if layout == LAYOUT_GEMV else round_up(K, 16)
    codes = torch.empty(M, ld, device=device, dtype=torch.int8)
    inv = torch.empty(M, device=device, dtype=torch.float32)
    rowsum = torch.empty(M, device=device, dtype=torch.int32) if layout == LAYOUT_GEMV else None
    return QuantAct(codes, inv, rowsum, layout, M)


def quantize(x2d: torch.Tensor, eps: float) -> QuantAct:
    M = x2d.shape[0]
    layout = layout_for(M)
    codes, inv, rowsum = quant_act(x2d, eps, layout)
    return QuantAct(codes, inv, rowsum, layout, M)


def matmul_q(q: QuantAct, pw: PackedWeight, out_dtype: torch.dtype, out=None):
    if q.layout == LAYOUT_GEMV:
        return gemv(q.codes, q.inv, q.rowsum, pw, q.M, out_dtype, out)
    return gemm(q.codes, q.inv, pw, q.M, out_dtype, out)


def pack_into(w: torch.Tensor, eps: float, packed: torch.Tensor, tern: Optional[torch.Tensor],
              scale: torch.Tensor, deq: torch.Tensor):
    """Pack one weight into caller-provided row slices (used to fuse gate/up weights)."""
    N, K = w.shape
    work = torch.empty(N, device=w.device, dtype=torch.float64)
    _lib.call("tesm_b200_weight_scale", w.data_ptr(), dtype_code(w.dtype), N, K, w.stride(0), 0, float(eps),
              scale.data_ptr(), deq.data_ptr(), work.data_ptr(), _stream())
    _lib.call("tesm_b200_pack_ternary", w.data_ptr(), dtype_code(w.dtype), N, K, w.stride(0), 0, scale.data_ptr(),
              packed.data_ptr(), packed.stride(0), _ptr(tern), tern.stride(0) if tern is not None else 0, _stream())


# ------------------------------------------------------------------ layer kernels
def scan_workspace(B: int, L: int, C: int, RM: int, device) -> torch.Tensor:
    n = ctypes.c_int64(0)
    _lib.call("tesm_b200_scan_workspace", B, L, C, RM, ctypes.addressof(n))
    return torch.empty(n.value, device=device, dtype=torch.uint8)


def siso_scan(proj, B, L, Dm, D, R, decay_bias, h0, states, f32, f64, scan_chunk=16):
    """SISO scan; ``scan_chunk`` is the module's state_scan_chunk_size (the reference's chunked
    fp64 formula clamps the in-chunk decay product at 1e-12, which the kernel reproduces)."""
    ws = scan_workspace(B, L, D, 1, proj.device)
    _lib.call("tesm_b200_siso_scan", proj.data_ptr(), dtype_code(proj.dtype), proj.stride(0), B, L, Dm, D, R,
              int(scan_chunk), decay_bias.data_ptr(), _ptr(h0), states.data_ptr(), f32.data_ptr(), f64.data_ptr(), ws.data_ptr(),
              ws.numel(), _stream())


def mimo_scan(proj, B, L, Dm, H, D, R, RM, decay_bias, mimo_x, states, f32, f64):
    ws = scan_workspace(B, L, H * D, RM, proj.device)
    _lib.call("tesm_b200_mimo_scan", proj.data_ptr(), dtype_code(proj.dtype), proj.stride(0), B, L, Dm, H, D, R, RM,
              decay_bias.data_ptr(), mimo_x.data_ptr(), states.data_ptr(), f32.data_ptr(), f64.data_ptr(),
              ws.data_ptr(), ws.numel(), _stream())


def siso_local_ent(proj, B, L, Dm, D, R, W, cross, bias, states, thr, es, base, out_tanh, out_chg):
    _lib.call("tesm_b200_siso_local_ent", proj.data_ptr(), dtype_code(proj.dtype), proj.stride(0), B, L, Dm, D, R, W,
              _ptr(cross), bias.data_ptr(), states.data_ptr(), float(thr), float(es), float(base),
              out_tanh.data_ptr(), out_chg.data_ptr(), dtype_code(out_tanh.dtype), _stream())


def global_relbias(embed, scale, bias0, L):
    out = torch.empty(2 * L - 1, device=embed.device, dtype=torch.float32)
    _lib.call("tesm_b200_global_relbias", embed.data_ptr(), embed.numel(), float(scale), float(bias0), L,
              out.data_ptr(), _stream())
    return out


def global_ent_tc_ok(D, R):
    return R <= 64 and R % 2 == 0 and D <= 256


def siso_global_ent(proj, B, L, Dm, D, R, cross, relb, states, thr, es, base, out_tanh, out_chg, force=None):
    """Causal global entanglement: tensor-core kernel when ent_rank <= 64 and d_state <= 256
    (force="tc" / "simt" picks one for tests), else the fp32 SIMT kernel."""
    path = force or ("tc" if global_ent_tc_ok(D, R) else "simt")
    if path == "tc":
        n = ctypes.c_int64(0)
        _lib.call("tesm_b200_global_ent_tc_workspace", B, L, D, R, ctypes.addressof(n))
        raw = torch.empty(n.value + 1024, device=proj.device, dtype=torch.uint8)
        off = (-raw.data_ptr()) % 1024  # 1024-byte aligned start
        _lib.call("tesm_b200_siso_global_ent_tc", proj.data_ptr(), dtype_code(proj.dtype), proj.stride(0), B, L, Dm,
                  D, R, _ptr(cross), relb.data_ptr(), states.data_ptr(), float(thr), float(es), float(base),
                  out_tanh.data_ptr(), out_chg.data_ptr(), dtype_code(out_tanh.dtype), raw.data_ptr() + off,
                  n.value, _stream())
        return
    _lib.call("tesm_b200_siso_global_ent", proj.data_ptr(), dtype_code(proj.dtype), proj.stride(0), B, L, Dm, D, R,
              _ptr(cross), relb.data_ptr(), states.data_ptr(), float(thr), float(es), float(base),
              out_tanh.data_ptr(), out_chg.data_ptr(), dtype_code(out_tanh.dtype), _stream())


def mimo_local_ent(proj, B, L, Dm, H, D, R, RM, W, bias, mimo_o, states, thr, es, base, quirk, out_tanh, out_chg):
    _lib.call("tesm_b200_mimo_local_ent", proj.data_ptr(), dtype_code(proj.dtype), proj.stride(0), B, L, Dm, H, D, R,
              RM, W, bias.data_ptr(), mimo_o.data_ptr(), states.data_ptr(), float(thr), float(es), float(base),
              int(quirk), out_tanh.data_ptr(), out_chg.data_ptr(), dtype_code(out_tanh.dtype), _stream())


def combine(proj, M, Dm, C, Rc, sp, ep, y):
    _lib.call("tesm_b200_combine", proj.data_ptr(), dtype_code(proj.dtype), proj.stride(0), M, Dm, C, Rc,
              sp.data_ptr(), ep.data_ptr(), dtype_code(sp.dtype), y.data_ptr(), dtype_code(y.dtype), _stream())


def cache_fill(proj, states, RM, B, L, Dm, H, D, R, W, base, final64, state, kc, vc, ctl):
    _lib.call("tesm_b200_cache_fill", proj.data_ptr(), dtype_code(proj.dtype), proj.stride(0), states.data_ptr(), RM,
              B, L, Dm, H, D, R, W, float(base), final64.data_ptr(), state.data_ptr(), kc.data_ptr(), vc.data_ptr(),
              ctl.data_ptr(), _stream())


def decode_step(proj, B, Dm, H, D, R, W, decay_bias, bias, cross, state, kc, vc, ctl, thr, es, base, out_tanh,
                out_chg, new_state):
    _lib.call("tesm_b200_decode_step", proj.data_ptr(), dtype_code(proj.dtype), proj.stride(0), B, Dm, H, D, R, W,
              decay_bias.data_ptr(), bias.data_ptr(), _ptr(cross), state.data_ptr(), kc.data_ptr(), vc.data_ptr(),
              ctl.data_ptr(), float(thr), float(es), float(base), out_tanh.data_ptr(), out_chg.data_ptr(),
              dtype_code(out_tanh.dtype), _ptr(new_state), _stream())


def siso_decode_step_codes(proj, B, Dm, D, R, W, decay_bias, bias, cross, state, kc, vc, ctl, thr, es, base,
                           act_dtype, eps1, eps2, new_state, xstate=None, xq: Optional[PackedWeight] = None,
                           xq_eps=0.0):
    """One-token SISO step emitting the int8 codes of tanh(ent) | ent - s for the combine GEMM.
    With ``xstate`` (the previous layer's fp32 state, (B, D)) and ``xq`` (cross_layer_q_proj's
    packed weight) the step computes the cross-layer query bias itself."""
    Dp = round_up(D, 128)
    codes = torch.empty(B, 2 * Dp, device=proj.device, dtype=torch.int8)
    inv1 = torch.empty(B, device=proj.device, dtype=torch.float32)
    inv2 = torch.empty(B, device=proj.device, dtype=torch.float32)
    _lib.call("tesm_b200_siso_decode_step_codes", proj.data_ptr(), dtype_code(proj.dtype), proj.stride(0), B, Dm, D,
              R, W, decay_bias.data_ptr(), bias.data_ptr(), _ptr(cross), state.data_ptr(), kc.data_ptr(),
              vc.data_ptr(), ctl.data_ptr(), float(thr), float(es), float(base), dtype_code(act_dtype), float(eps1),
              float(eps2), codes.data_ptr(), codes.stride(0), Dp, inv1.data_ptr(), inv2.data_ptr(), _ptr(new_state),
              _ptr(xstate), _ptr(xq.tern) if xq is not None else None, xq.tern.stride(0) if xq is not None else 0,
              _ptr(xq.deq) if xq is not None else None, float(xq_eps), _stream())
    return codes, inv1, inv2, Dp


def embed(ids, emb, pos_emb, pos_dev, pos_host, out):
    B, L = ids.shape
    _lib.call("tesm_b200_embed", ids.data_ptr(), B, L, emb.data_ptr(), pos_emb.data_ptr(), dtype_code(emb.dtype),
              emb.shape[1], _ptr(pos_dev), int(pos_host), out.data_ptr(), dtype_code(out.dtype), _stream())


def add_rmsnorm_quant(x, residual, residual_out, weight, eps, qeps, q: Optional[QuantAct], y_out=None):
    M, K = x.shape
    _lib.call("tesm_b200_add_rmsnorm_quant", x.data_ptr(), dtype_code(x.dtype), _ptr(residual), _ptr(residual_out),
              weight.data_ptr(), float(eps), M, K, float(qeps), _ptr(q.codes) if q else None,
              q.codes.stride(0) if q else 0, q.layout if q else 0, _ptr(q.inv) if q else None,
              _ptr(q.rowsum) if q else None, _ptr(y_out), dtype_code(y_out.dtype) if y_out is not None else 0,
              _stream())


def silu_mul(gu, F, out, blk=0):
    _lib.call("tesm_b200_silu_mul", gu.data_ptr(), dtype_code(gu.dtype), gu.shape[0], F, blk, out.data_ptr(),
              dtype_code(out.dtype), _stream())


_SWIGLU_WIDE = os.environ.get("TESM_SKINNY_WIDE", "1") != "0"


def gemm_swiglu(q: QuantAct, pw: PackedWeight, out_dtype, out=None):
    """Interleaved gate/up weight (blocks of 128 rows) -> silu(gate) * up, width pw.N // 2."""
    F = pw.N // 2
    out = out if out is not None else torch.empty(q.M, F, device=q.codes.device, dtype=out_dtype)
    if q.M <= 128 or (q.M <= 256 and not _SWIGLU_WIDE):
        # small batches: skinny-tile GEMM, then the gate on the interleaved output
        gu = gemm(q.codes, q.inv, pw, q.M, out_dtype)
        silu_mul(gu, F, out, 128)
        return out
    ws = splitk_workspace(q.M, pw.N, q.codes.device)
    _lib.call("tesm_b200_gemm_i8_swiglu", q.codes.data_ptr(), q.codes.stride(0), q.inv.data_ptr(), pw.tern.data_ptr(),
              pw.tern.stride(0), pw.deq.data_ptr(), q.M, F, pw.K, out.data_ptr(), dtype_code(out.dtype),
              out.stride(0), _ptr(ws), ws.numel() * 4 if ws is not None else 0, _stream())
    return out


def device_status() -> int:
    v = ctypes.c_int(0)
    _lib.call("tesm_b200_device_status", ctypes.addressof(v))
    return v.value



def siso_local_ent_codes(proj, B, L, Dm, D, R, W, cross, bias, states, thr, es, base, act_dtype, eps1, eps2):
    """Local entanglement emitting the int8 codes of tanh(ent) | ent - s (see the C header)."""
    Dp = round_up(D, 128)
    M = B * L
    codes = torch.empty(M, 2 * Dp, device=proj.device, dtype=torch.int8)
    inv1 = torch.empty(M, device=proj.device, dtype=torch.float32)
    inv2 = torch.empty(M, device=proj.device, dtype=torch.float32)
    _lib.call("tesm_b200_siso_local_ent_codes", proj.data_ptr(), dtype_code(proj.dtype), proj.stride(0), B, L, Dm, D,
              R, W, _ptr(cross), bias.data_ptr(), states.data_ptr(), float(thr), float(es), float(base),
              dtype_code(act_dtype), float(eps1), float(eps2), codes.data_ptr(), codes.stride(0), Dp,
              inv1.data_ptr(), inv2.data_ptr(), _stream())
    return codes, inv1, inv2, Dp


def gemm_combine(codes, Kh, inv1, inv2, tern, deq1, deq2, proj, c_local, c_gate, M, N, out):
    _lib.call("tesm_b200_gemm_i8_combine", codes.data_ptr(), codes.stride(0), Kh, inv1.data_ptr(), inv2.data_ptr(),
              tern.data_ptr(), tern.stride(0), deq1.data_ptr(), deq2.data_ptr(), proj.data_ptr(),
              dtype_code(proj.dtype), proj.stride(0), c_local, c_gate, M, N, out.data_ptr(), dtype_code(out.dtype),
              out.stride(0), _stream())
    return out


def mimo_global_ent(proj, B, L, Dm, H, D, R, RM, relb, mimo_o, states, thr, base, out_tanh, out_chg):
    acc_e = acc_c = None
    if RM > 1:
        acc_e = torch.empty(B * L, H * D, device=proj.device, dtype=torch.float32)
        acc_c = torch.empty_like(acc_e)
    _lib.call("tesm_b200_mimo_global_ent", proj.data_ptr(), dtype_code(proj.dtype), proj.stride(0), B, L, Dm, H, D,
              R, RM, relb.data_ptr(), mimo_o.data_ptr(), states.data_ptr(), float(thr), float(base), _ptr(acc_e),
              _ptr(acc_c), out_tanh.data_ptr(), out_chg.data_ptr(), dtype_code(out_tanh.dtype), _stream())
