// One-token incremental step of a TESM layer against its recurrent-state cache.
// SISO: TESM_SISO._forward_incremental (tesm.py:1274-1400); MIMO (H heads, no rank mixing):
// TESMMIMO_Optimized._forward_incremental (tesm_mimo.py:753-912).
//
//  * new_state = a * state + w * tanh(v) in fp64, state kept in fp64 like the reference;
//  * ring write of (rope(k), new_state as fp32) at slot cache_idx, then cache_idx advances;
//  * window order follows the reference exactly: a full window is gathered from slot
//    cache_idx (the entry just written) onward with bias[w]; a partial window reads slots
//    [0, valid) with bias[W - valid + w];
//  * ternary, normalised signed average, lerp -> tanh(ent) and ent - new_state.
// seq_pos / cache_idx live in a device int pair so a captured CUDA graph can replay steps;
// the last CTA to finish advances them (every CTA reads them before it increments the
// completion counter, so no CTA can observe the advanced values).
#include "layer_common.cuh"
#include "rowio.cuh"

namespace tesm {

struct DecodeParams {
  ProjCols pc;                // (B, Nproj)
  const float *decay_bias;    // (H*D)
  const float *bias;          // (H, W)
  const float *cross;         // (B, H*R) or null
  double *state;              // (B, H, D)
  float *kc;                  // (B, W, H, R)
  float *vc;                  // (B, W, H, D)
  int *ctl;                   // [seq_pos, cache_idx, done_counter]
  int B, H, D, R, W;
  float thr, es, sqrt_r, rope_base;
  RopeTab rt;
  void *out_tanh, *out_chg;   // (B, H*D)
  int out_dtype;
  float *new_state;           // (B, H*D) fp32 (cross-layer state for the next layer)
  // codes mode (SISO, one block per row): instead of tanh(ent) / ent - s, their per-token int8
  // codes (values first rounded to act_dtype, as the BitLinear input quantiser sees them) in
  // the combine GEMM's A layout: tanh codes in [0, D), change codes in [Dp, Dp + D)
  int8_t *codes;
  int64_t ldc;
  int Dp, act_dtype;
  float eps1, eps2;
  float *inv1, *inv2;
  // fused cross-layer query bias (SISO, one block per row): cross = BitLinear(xstate[row]) with
  // the fp32 input quantised per row and the int8 ternary weight xq_t (R rows, pitch xq_ld);
  // replaces `cross` when xstate is set
  const float *xstate;  // (B, D) fp32: the previous layer's new state
  const int8_t *xq_t;
  int64_t xq_ld;
  const float *xq_deq;
  float xq_eps;
};

// Cross-layer query bias of one row, as BitLinear (tesm.py:206-215, 287-290) on the fp32
// state row: per-row int8 codes (the activation quantiser of quant.cu), exact int32 dot products
// with the ternary rows (4 threads per output, dp4a over 16-byte groups), dequantised as
// (float)acc * (1/s) * deq like the BitLinear GEMM / GEMV epilogues.  blockDim >= D.
__device__ void cross_bias_row(const DecodeParams &p, int64_t row, int8_t *xc, float *out, float *red) {
  const int tid = threadIdx.x, D = p.D, Dk = (D + 15) & ~15;
  const float x = tid < D ? p.xstate[row * D + tid] : 0.f;
  const float amax = block_reduce(fabsf(x), red, [](float a, float b) { return fmaxf(a, b); }, 0.f);
  const float s = act_scale(amax, p.xq_eps, TESM_F32);
  if (tid < Dk) xc[tid] = tid < D ? (int8_t)act_code(x, s, TESM_F32) : 0;
  for (int i = tid + blockDim.x; i < Dk; i += blockDim.x) xc[i] = 0;
  __syncthreads();
  const float inv = __frcp_rn(s), wd = p.xq_deq[0];
  const int groups = Dk / 16;
  for (int o0 = 0; o0 < p.R; o0 += blockDim.x / 4) {
    const int o = o0 + tid / 4, part = tid & 3;
    int acc = 0;
    if (o < p.R) {
      const int8_t *wr = p.xq_t + (int64_t)o * p.xq_ld;
      for (int g = part; g < groups; g += 4) {
        const int4 w4 = *reinterpret_cast<const int4 *>(wr + g * 16);
        const int4 c4 = *reinterpret_cast<const int4 *>(xc + g * 16);
        acc = __dp4a(w4.x, c4.x, acc);
        acc = __dp4a(w4.y, c4.y, acc);
        acc = __dp4a(w4.z, c4.z, acc);
        acc = __dp4a(w4.w, c4.w, acc);
      }
    }
    acc += __shfl_xor_sync(0xffffffffu, acc, 1);
    acc += __shfl_xor_sync(0xffffffffu, acc, 2);
    if (o < p.R && part == 0) out[o] = (float)acc * inv * wd;
  }
  __syncthreads();
}

__global__ void k_decode_step(const __grid_constant__ DecodeParams p) {
  extern __shared__ float sm[];
  pdl_trigger();
  pdl_wait();
  const int R = p.R, W = p.W, D = p.D, H = p.H;
  float *q = sm;             // R
  float *k = q + R;          // R
  float *tw = k + R;         // W weights (ternary / norm)
  int *slot = reinterpret_cast<int *>(tw + W);  // W
  float *xb = reinterpret_cast<float *>(slot + W);          // R: fused cross-layer bias
  int8_t *xc = reinterpret_cast<int8_t *>(xb + R);          // D rounded up to 16: its input codes
  const int h = blockIdx.x, b = blockIdx.y;
  const int pos = p.ctl[0], idx = p.ctl[1];
  const int valid = min(pos + 1, W);
  const int64_t row = b;
  const int C = H * D;
  const int tid = threadIdx.x;
  if (p.xstate) {
    __shared__ float xred[32];
    cross_bias_row(p, row, xc, xb, xred);
  }
  load_rope_row(q, p.pc, p.pc.c_q + h * R, row, R, pos, p.rt.v,
                p.xstate ? xb : (p.cross ? p.cross + row * H * R + h * R : nullptr), tid, blockDim.x);
  load_rope_row(k, p.pc, p.pc.c_k + h * R, row, R, pos, p.rt.v, nullptr, tid, blockDim.x);
  __syncthreads();
  float *kslot = p.kc + (((int64_t)b * W + idx) * H + h) * R;
  for (int i = tid; i < R; i += blockDim.x) kslot[i] = k[i];
  double newd = 0.0;
  for (int d = tid; d < D; d += blockDim.x) {  // blockDim >= D
    const int c = h * D + d;
    const float a = sigmoidf_(load_f(p.pc.proj, p.pc.dtype, row * p.pc.ld + p.pc.c_decay + c) + p.decay_bias[c]);
    const float w = sigmoidf_(load_f(p.pc.proj, p.pc.dtype, row * p.pc.ld + p.pc.c_write + c));
    const float v = tanhf(load_f(p.pc.proj, p.pc.dtype, row * p.pc.ld + p.pc.c_value + c));
    const int64_t si = ((int64_t)b * H + h) * D + d;
    newd = (double)a * p.state[si] + (double)w * (double)v;
    p.vc[(((int64_t)b * W + idx) * H + h) * D + d] = (float)newd;
  }
  __syncthreads();  // the slot just written is read back below
  // window scores: all W lags at once, 8 lanes per lag (W <= 32 needs blockDim >= 8*W, else a
  // second pass), partial dot products combined with shuffles within each 8-lane group
  for (int w0 = 0; w0 < W; w0 += blockDim.x / 8) {
    const int w = w0 + tid / 8, part_i = tid & 7;
    float part = 0.f;
    if (w < valid) {
      const int sl = valid >= W ? (idx + w) % W : w;
      const float *kr = p.kc + (((int64_t)b * W + sl) * H + h) * R;
      for (int i = part_i; i < R; i += 8) part = fmaf(q[i], kr[i], part);
    }
#pragma unroll
    for (int o = 4; o; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
    if (part_i == 0 && w < W) {
      float t = 0.f;
      if (w < valid) {
        const int bi = valid >= W ? w : W - valid + w;
        t = ternary_of(__fdiv_rn(part, p.sqrt_r) + p.bias[h * W + bi], p.thr);
      }
      tw[w] = t;
      slot[w] = w < valid ? (valid >= W ? (idx + w) % W : w) : 0;
    }
  }
  __syncthreads();
  if (tid < 32) {
    float cnt = tid < W ? fabsf(tw[tid]) : 0.f;
    cnt = warp_sum(cnt);
    if (tid < W) tw[tid] = tw[tid] / fmaxf(cnt, 1.f);
  }
  __syncthreads();
  float th = 0.f, cg = 0.f;  // this thread's channel (codes mode: d = tid, blockDim >= D)
  for (int d = tid; d < D; d += blockDim.x) {
    const int c = h * D + d;
    const float ns = (float)newd;
    float avg = 0.f;
    for (int w = 0; w < valid; ++w) avg = fmaf(tw[w], p.vc[(((int64_t)b * W + slot[w]) * H + h) * D + d], avg);
    const float ent = ns + p.es * (avg - ns);
    th = tanhf(ent);
    cg = ent - ns;
    if (!p.codes) {
      store_f(p.out_tanh, p.out_dtype, row * C + c, th);
      store_f(p.out_chg, p.out_dtype, row * C + c, cg);
    }
    p.state[((int64_t)b * H + h) * D + d] = newd;
    if (p.new_state) p.new_state[row * C + c] = ns;
  }
  if (p.codes) {  // per-token int8 codes of both outputs over the row (H == 1)
    __shared__ float red[32];
    const bool in = tid < D;
    th = round_to(p.act_dtype, in ? th : 0.f);
    cg = round_to(p.act_dtype, in ? cg : 0.f);
    const float a1 = block_reduce(fabsf(th), red, [](float x, float y) { return fmaxf(x, y); }, 0.f);
    const float a2 = block_reduce(fabsf(cg), red, [](float x, float y) { return fmaxf(x, y); }, 0.f);
    const float s1 = act_scale(a1, p.eps1, p.act_dtype), s2 = act_scale(a2, p.eps2, p.act_dtype);
    int8_t *crow = p.codes + row * p.ldc;
    for (int d = tid; d < p.Dp; d += blockDim.x) {  // zero padding up to Dp
      crow[d] = d < D ? (int8_t)act_code(th, s1, p.act_dtype) : 0;
      crow[p.Dp + d] = d < D ? (int8_t)act_code(cg, s2, p.act_dtype) : 0;
    }
    if (tid == 0) {
      p.inv1[row] = __frcp_rn(s1);
      p.inv2[row] = __frcp_rn(s2);
    }
  }
  // completion: the last CTA advances (seq_pos, cache_idx)
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    const int done = atomicAdd(&p.ctl[2], 1);
    if (done == (int)(gridDim.x * gridDim.y) - 1) {
      p.ctl[0] = pos + 1;
      p.ctl[1] = (idx + 1) % W;
      p.ctl[2] = 0;
      __threadfence();
    }
  }
}

}  // namespace tesm

using namespace tesm;

extern "C" int tesm_b200_decode_step(const void *proj, int dtype, int64_t ldp, int64_t B, int64_t Dm, int64_t H,
                                     int64_t D, int64_t R, int64_t W, const float *decay_bias, const float *bias,
                                     const float *cross, double *state, float *k_cache, float *v_cache, int *ctl,
                                     float thr, float es, float rope_base, void *out_tanh, void *out_chg,
                                     int out_dtype, float *new_state, tesm_stream_t stream) {
  TESM_REQUIRE(proj && decay_bias && bias && state && k_cache && v_cache && ctl && out_tanh && out_chg,
               "decode_step: null pointer");
  TESM_REQUIRE(B > 0 && H > 0 && D > 0 && D <= 1024 && R > 0 && R % 2 == 0 && W > 0 && W <= 32,
               "decode_step: bad shape (D <= 1024, W <= 32, even R)");
  if (dtype != TESM_F32 && dtype != TESM_BF16) return fail(TESM_EDTYPE, "decode_step: dtype");
  DecodeParams p = {};
  p.pc = make_cols(proj, dtype, ldp, (int)Dm, (int)(H * D), (int)(H * R));
  p.decay_bias = decay_bias;
  p.bias = bias;
  p.cross = cross;
  p.state = state;
  p.kc = k_cache;
  p.vc = v_cache;
  p.ctl = ctl;
  p.B = (int)B;
  p.H = (int)H;
  p.D = (int)D;
  p.R = (int)R;
  p.W = (int)W;
  p.thr = thr;
  p.es = es;
  p.sqrt_r = (float)sqrt((double)R);
  p.rope_base = rope_base;
  TESM_REQUIRE(R <= 256, "decode_step: ent_rank above 256");
  p.rt = rope_table((int)R, rope_base);
  p.out_tanh = out_tanh;
  p.out_chg = out_chg;
  p.out_dtype = out_dtype;
  p.new_state = new_state;
  p.codes = nullptr;
  const int threads = (int)round_up(D < 32 ? 32 : D, 32);
  const size_t smem = sizeof(float) * (2 * R + W) + sizeof(int) * W;
  dim3 grid((unsigned)H, (unsigned)B);
  return launch_k("decode_step", k_decode_step, grid, dim3(threads), smem, (cudaStream_t)stream, p);
}

extern "C" int tesm_b200_siso_decode_step_codes(const void *proj, int dtype, int64_t ldp, int64_t B, int64_t Dm,
                                                int64_t D, int64_t R, int64_t W, const float *decay_bias,
                                                const float *bias, const float *cross, double *state,
                                                float *k_cache, float *v_cache, int *ctl, float thr, float es,
                                                float rope_base, int act_dtype, float eps1, float eps2,
                                                int8_t *codes, int64_t ldc, int64_t Dp, float *inv1, float *inv2,
                                                float *new_state, const float *xstate, const int8_t *xq_tern,
                                                int64_t xq_ld, const float *xq_deq, float xq_eps,
                                                tesm_stream_t stream) {
  TESM_REQUIRE(proj && decay_bias && bias && state && k_cache && v_cache && ctl && codes && inv1 && inv2,
               "decode_step_codes: null pointer");
  TESM_REQUIRE(B > 0 && D > 0 && D <= 1024 && R > 0 && R % 2 == 0 && W > 0 && W <= 32,
               "decode_step_codes: bad shape (D <= 1024, W <= 32, even R)");
  TESM_REQUIRE(Dp >= D && Dp % 128 == 0 && ldc >= 2 * Dp, "decode_step_codes: Dp must be D rounded up to 128");
  if (dtype != TESM_F32 && dtype != TESM_BF16) return fail(TESM_EDTYPE, "decode_step_codes: dtype");
  if (act_dtype != TESM_F32 && act_dtype != TESM_BF16) return fail(TESM_EDTYPE, "decode_step_codes: act dtype");
  if (xstate)
    TESM_REQUIRE(xq_tern && xq_deq && xq_ld >= round_up(D, 16) && xq_ld % 16 == 0 && ((uintptr_t)xq_tern & 15) == 0,
                 "decode_step_codes: cross-layer weight must be int8 rows of >= D rounded up to 16 bytes, "
                 "16-byte aligned");
  DecodeParams p = {};
  p.pc = make_cols(proj, dtype, ldp, (int)Dm, (int)D, (int)R);
  p.decay_bias = decay_bias;
  p.bias = bias;
  p.cross = cross;
  p.state = state;
  p.kc = k_cache;
  p.vc = v_cache;
  p.ctl = ctl;
  p.B = (int)B;
  p.H = 1;
  p.D = (int)D;
  p.R = (int)R;
  p.W = (int)W;
  p.thr = thr;
  p.es = es;
  p.sqrt_r = (float)sqrt((double)R);
  p.rope_base = rope_base;
  TESM_REQUIRE(R <= 256, "decode_step: ent_rank above 256");
  p.rt = rope_table((int)R, rope_base);
  p.out_tanh = p.out_chg = nullptr;
  p.out_dtype = act_dtype;
  p.new_state = new_state;
  p.codes = codes;
  p.ldc = ldc;
  p.Dp = (int)Dp;
  p.act_dtype = act_dtype;
  p.eps1 = eps1;
  p.eps2 = eps2;
  p.inv1 = inv1;
  p.inv2 = inv2;
  p.xstate = xstate;
  p.xq_t = xq_tern;
  p.xq_ld = xq_ld;
  p.xq_deq = xq_deq;
  p.xq_eps = xq_eps;
  const int threads = (int)round_up(D < 32 ? 32 : D, 32);
  const size_t smem = sizeof(float) * (3 * R + W) + sizeof(int) * W + (size_t)round_up(D, 16);
  return launch_k("decode_step_codes", k_decode_step, dim3(1, (unsigned)B), dim3(threads), smem,
                  (cudaStream_t)stream, p);
}
