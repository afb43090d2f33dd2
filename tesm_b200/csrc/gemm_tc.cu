// Prefill-shaped int8 GEMM on the sm_100a tensor cores:
//   D[m,n] = sum_k A[m,k] * B[n,k]      (A: activation codes, B: ternary weights, int32 exact)
//   out[m,n] = D * inv_scale[m] * w_deq[n|0]
//
// Persistent, warp-specialised CTA (one per SM, 320 threads):
//   warp 0     : TMA producer (one elected thread), 128-byte swizzled K-major tiles,
//                STAGES-deep smem ring guarded by full/empty mbarriers;
//   warp 1     : TMEM allocator + MMA issuer (one thread): tcgen05.mma.cta_group::1.kind::i8,
//                M=128 x N=BN x K=32 per instruction, accumulator in TMEM, double-buffered
//                across output tiles so the epilogue of tile i overlaps the MMAs of tile i+1;
//   warps 2..9 : epilogue: tcgen05.ld 32 lanes x 32 columns, scale, convert, store; warp w
//                reads TMEM lanes 32*(w%4).. and half of the tile's columns.
// Every mbarrier wait is bounded; a wait that gives up sets the sticky device status
// (TESM_ETIMEOUT) and the CTA drains and exits instead of hanging.
#include "rowio.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstdlib>
#include <mutex>
#include <unordered_map>

namespace tesm {

namespace tc {

constexpr int BM = 128;
constexpr int BK = 128;  // bytes (= int8 elements) per k-block: one 128B swizzle atom
constexpr int STAGES = 4;
constexpr int EPI_WARPS = 8;  // two epilogue warps per TMEM lane quarter, splitting the columns
constexpr int NUM_THREADS = 64 + 32 * EPI_WARPS;
constexpr long long kWaitCycles = 4000000000ll;  // ~2 s at B200 clocks

struct Params {
  const float *inv_scale;
  const float *w_deq;
  int per_row;
  int M, N, K;
  void *out;
  int out_dtype;
  int64_t ldo;
  int32_t *acc_out;
  int64_t ld_acc;
  int num_m_tiles, num_n_tiles, num_k_blocks, group_m;
  int vec_store;
  int swiglu;  // 1: weight rows interleaved [128 gate | 128 up] per tile; out = silu(g) * u, width N/2
  // dual-accumulator combine (DUAL kernels): k-blocks [0, ksplit) accumulate acc1, the rest acc2;
  // out = local + sigmoid(gate) * acc1*inv_scale*w_deq[0] + acc2*inv_scale2*w_deq2[0]
  int ksplit;
  const float *inv_scale2;
  const float *w_deq2;
  const void *proj;
  int proj_dtype;
  int64_t ldp;
  int c_local, c_gate;
  int proj_vec;
  int dual_tma;  // bf16 proj and output, 16-byte aligned: local/gate via TMA loads, output via TMA store
  // split-K (small M).  Work units: the first n_full tiles whole, then every remaining tile
  // cut into `splits` k-ranges, all of them in one round of the persistent loop.  A split owns
  // the 32-column chunks c with c % splits == its index: it stores its int32 partials of the
  // other chunks into its slice of `part`, counts itself in cnt[tile * 2 + pair rank], waits
  // until every split has counted, adds the other slices to its own chunks (exact integers)
  // and runs the epilogue on them; a second count resets the counter to zero for the next call.
  int splits, n_full;
  int pdl_late;  // 1: signal dependents when the epilogue starts the CTA's last unit (else at entry)
  int32_t *ws;      // caller scratch: kCounterInts counters (zero between calls), then the slices
  int64_t ws_bytes;
  int32_t *cnt, *part;
  int part_rb, part_cb;  // 32-row blocks and 32-column blocks of one partial slice
};

constexpr int kCounterInts = 4096;  // 16 KB of tile counters at the start of the split-K scratch


// work unit u -> (tile, split, number of splits of that tile)
__device__ __forceinline__ void unit_info(const Params &p, int u, int &t, int &sp, int &ns) {
  if (u < p.n_full) {
    t = u;
    sp = 0;
    ns = 1;
  } else {
    const int v = u - p.n_full;
    t = p.n_full + v / p.splits;
    sp = v - (t - p.n_full) * p.splits;
    ns = p.splits;
  }
}

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

// release / acquire at CTA and GPU scope for the split-K meeting
__device__ __forceinline__ void red_release_cta(int *a, int v) {
  asm volatile("red.release.cta.shared::cta.add.s32 [%0], %1;\n" ::"r"(smem_u32(a)), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_cta(const int *a) {
  int v;
  asm volatile("ld.acquire.cta.shared::cta.b32 %0, [%1];\n" : "=r"(v) : "r"(smem_u32(a)) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_cta(int *a, int v) {
  asm volatile("st.release.cta.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(a)), "r"(v) : "memory");
}
__device__ __forceinline__ void red_release_gpu(int *a, int v) {
  asm volatile("red.release.gpu.global.add.s32 [%0], %1;\n" ::"l"(a), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_gpu(const int *a) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];\n" : "=r"(v) : "l"(a) : "memory");
  return v;
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(bytes));
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(smem_u32(bar)));
}

// Bounded parity wait. Returns false (after flagging the device status) on timeout.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity) {
  const uint32_t addr = smem_u32(bar);
  const long long t0 = clock64();
  while (true) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(addr), "r"(parity)
        : "memory");
    if (ok) return true;
    if (clock64() - t0 > kWaitCycles) {
      flag_timeout();
      return false;
    }
  }
}

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, uint64_t *bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];\n" ::"r"(
          smem_u32(dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// ---- CTA pairs (cta_group::2): one M=256 MMA over two SMs, each holding half of A and B ----
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;\n" : "=r"(r));
  return r;
}
// address of the same shared-memory variable in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;\n" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release;\nbarrier.cluster.wait.acquire;\n" ::: "memory");
}
// TMA load into this CTA's shared memory whose completion is counted on the pair leader's
// barrier (bar_cluster: a shared::cluster address).  No multicast.
__device__ __forceinline__ void tma_load_2d_pair(void *dst, const CUtensorMap *map, uint32_t bar_cluster, int x,
                                                 int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, "
      "%4}], [%2];\n" ::"r"(smem_u32(dst)),
      "l"(map), "r"(bar_cluster), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar_cluster) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];\n" ::"r"(bar_cluster) : "memory");
}

// K-major operand tile with 128-byte swizzle: 8-row atoms 1024 B apart (SBO), version 1.
__device__ __forceinline__ uint64_t smem_desc_sw128(const void *p) {
  const uint64_t addr = smem_u32(p);
  return ((addr >> 4) & 0x3FFFull) | (1ull << 16) | (64ull << 32) | (1ull << 46) | (2ull << 61);
}

// kind::i8 instruction descriptor: D s32, A/B signed int8, both K-major, M=m (128, or 256 for
// a CTA pair), N=n.
__host__ __device__ constexpr uint32_t idesc_i8(int n, int m = BM) {
  return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

// kind::f16 with bf16 operands and an fp32 accumulator (the dense lm_head).
__host__ __device__ constexpr uint32_t idesc_bf16(int n, int m = BM) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ void mma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void mma_bf16_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                              uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void mma_i8_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

// Completion of the pair's MMAs signalled on the barrier at this offset in both CTAs.
__device__ __forceinline__ void mma_commit_pair(uint64_t *bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;\n" ::"r"(
          smem_u32(bar)),
      "h"((uint16_t)3)
      : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory"); }

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
}

// TMA store of a shared-memory tile (bulk-group completion), and the group waits.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap *map, const void *src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];\n" ::"l"(map),
               "r"(smem_u32(src)), "r"(x), "r"(y)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;\n" ::"n"(N) : "memory");
}
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;\n" ::: "memory"); }
// generic-proxy shared-memory writes -> visible to a following TMA (async proxy) read
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
}
__device__ __forceinline__ uint4 lds128(uint32_t saddr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];\n" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(saddr));
  return v;
}

// int32 accumulator -> float without the conversion unit (shared with the transcendentals):
// for |a| < 2^22, 1.5*2^23 + a is exact in fp32 and its bit pattern is 0x4B400000 + a.  The
// combine GEMM guarantees the bound (|a| <= 128 * Kh with Kh <= 16384).
__device__ __forceinline__ float acc_to_f(uint32_t a) {
  return __int_as_float((int)a + 0x4B400000) - 12582912.f;
}
// Sigmoid for the combine epilogue: two transcendental-unit ops (exp2, approximate reciprocal),
// relative error a few ulp; exp overflow gives 1/inf = 0, the correct limit.
__device__ __forceinline__ float epi_sigmoid(float x) { return __fdividef(1.f, 1.f + __expf(-x)); }
// The output combine of the dual-accumulator epilogue, local + sigmoid(gate) * sp + ep with
// sp = acc1 * s1 and ep = acc2 * s2, as explicit fused multiply-adds so that every kernel that
// applies it (both epilogue variants, k_combine_acc) rounds identically.
__device__ __forceinline__ float combine_first(float loc, float gate, float a1, float s1) {
  return __fmaf_rn(epi_sigmoid(gate), __fmul_rn(a1, s1), loc);
}
__device__ __forceinline__ float combine_second(float v, float a2, float s2) { return __fmaf_rn(a2, s2, v); }

__device__ __forceinline__ void tile_coords(const Params &p, int t, int &mt, int &nt) {
  const int per_group = p.group_m * p.num_n_tiles;
  const int grp = t / per_group;
  const int first_m = grp * p.group_m;
  const int gm = min(p.num_m_tiles - first_m, p.group_m);
  const int r = t - grp * per_group;
  nt = r / gm;
  mt = first_m + (r - nt * gm);
}

// BF: bf16 operands (kind::f16, K counted in bytes, 64 elements per k-block), fp32 accumulators
// written unscaled (plain tiles only, no split-K).
template <int BN, bool DUAL, int MT, bool PAIR, bool BF = false>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    k_gemm_i8(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
              const __grid_constant__ CUtensorMap tmL, const __grid_constant__ CUtensorMap tmG,
              const __grid_constant__ CUtensorMap tmO, Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  // MT = 2 ("skinny", decode batches): one CTA covers 256 token rows as two M=128 MMAs sharing
  // each weight tile, so a narrow N tile still reads every weight byte once
  // PAIR: a cluster of two CTAs computes a 256-row tile with M=256 MMAs issued by the even CTA
  // (the leader); each CTA stages its own 128 rows of A and half (BN/2 rows) of the weight tile,
  // and holds its 128 accumulator rows in its own TMEM.
  static_assert(!PAIR || (MT == 1 && !DUAL), "CTA pairs: plain tiles only");
  constexpr int NST = PAIR ? 6 : STAGES;
  constexpr int A_BYTES = MT * BM * BK;
  constexpr int B_BYTES = (PAIR ? BN / 2 : BN) * BK;
  uint8_t *sA = smem;
  uint8_t *sB = smem + NST * A_BYTES;
  uint64_t *bars = reinterpret_cast<uint64_t *>(sB + NST * B_BYTES);
  uint64_t *full = bars, *empty = bars + NST, *tfull = bars + 2 * NST, *tempty = bars + 2 * NST + 2;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 2 * NST + 4);
  // DUAL with bf16 proj and output (p.dual_tma): per epilogue warp and 32-column chunk, the
  // 32x32 bf16 local and gate tiles (TMA loads, one mbarrier each) and the output tile (TMA
  // store), all with the 64-byte swizzle so lane-per-row accesses hit distinct banks.
  constexpr int DCH = DUAL ? BN / 64 : 1;  // 32-column chunks per epilogue warp
  uint64_t *pbar = bars + 2 * NST + 6;  // EPI_WARPS * DCH barriers
  uint8_t *sP = sB + NST * B_BYTES + 1024;  // 1024-aligned (swizzled TMA boxes)
  uint8_t *sO = sP + EPI_WARPS * DCH * 2 * 2048;
  // plain / SwiGLU epilogues: a 4 KB staging block per epilogue warp, through which each 32 x 32
  // output chunk is transposed so that global stores cover whole row segments
  uint8_t *sStage = sP;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t crank = PAIR ? cluster_rank() : 0;  // 0: the pair leader
  // persistent loop over work units: per CTA, or per CTA pair
  const int ustart = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
  const int ustride = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;
  constexpr uint32_t ACC_COLS = DUAL ? 2 * BN : MT * BN;  // TMEM columns of one tile's accumulator(s)
  constexpr uint32_t TMEM_COLS = 2 * ACC_COLS;

  // split-K meeting words of the epilogue warps (see the split-K branch of the epilogue)
  __shared__ int s_last, s_arrive, s_decided;
  if (threadIdx.x == 0) {
    s_last = s_arrive = s_decided = 0;
    for (int i = 0; i < NST; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], PAIR ? 2 * EPI_WARPS : EPI_WARPS);  // pair: both CTAs' epilogues
    }
    if (DUAL)
      for (int i = 0; i < EPI_WARPS * DCH; ++i) mbar_init(&pbar[i], 1);
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    asm volatile("prefetch.tensormap [%0];\n" ::"l"(&tmA) : "memory");
    asm volatile("prefetch.tensormap [%0];\n" ::"l"(&tmB) : "memory");
  }
  if (warp == 1) {
    if (PAIR) {  // both CTAs of the pair allocate together
      asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(
                       smem_u32(tmem_slot)),
                   "r"(TMEM_COLS));
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;\n");
    } else {
      asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(
                       smem_u32(tmem_slot)),
                   "r"(TMEM_COLS));
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n");
    }
  }
  fence_before();
  if (PAIR)
    cluster_sync();  // the peer's barriers are initialised before any remote arrive
  else
    __syncthreads();
  fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // programmatic dependent launch: the set-up above overlapped the previous kernel; only the
  // producer's first weight-tile requests (constant data) go out before its completion
  if (threadIdx.x == 0 && !p.pdl_late) pdl_trigger();
  if (warp != 0) pdl_wait();

  const int total = p.n_full + (p.num_m_tiles * p.num_n_tiles - p.n_full) * p.splits;
  const int nk_all = p.num_k_blocks;

  if (warp == 0) {
    if (lane == 0) {
      // weight tiles of the first stages: requested before waiting for the previous kernel
      int pre = 0;
      if (ustart < total) {
        int mt, nt, t, sp, ns;
        unit_info(p, ustart, t, sp, ns);
        tile_coords(p, t, mt, nt);
        const int kb_lo = sp * nk_all / ns, kb_hi = (sp + 1) * nk_all / ns;
        pre = kb_hi - kb_lo < NST ? kb_hi - kb_lo : NST;
        for (int i = 0; i < pre; ++i) {  // fresh stages: no empty-barrier wait needed
          const int kb = kb_lo + i;
          if (PAIR) {
            if (crank == 0) mbar_expect_tx(&full[i], 2 * (A_BYTES + B_BYTES));
            tma_load_2d_pair(sB + i * B_BYTES, &tmB, mapa_shared(smem_u32(&full[i]), 0), kb * BK,
                             nt * BN + (int)crank * (BN / 2));
          } else {
            mbar_expect_tx(&full[i], A_BYTES + B_BYTES);
            tma_load_2d(sB + i * B_BYTES, &tmB, &full[i], kb * BK, nt * BN);
          }
        }
      }
      pdl_wait();
      uint32_t it = 0;
      bool ok = true;
      for (int u = ustart; u < total && ok; u += ustride) {
        int mt, nt, t, sp, ns;
        unit_info(p, u, t, sp, ns);
        tile_coords(p, t, mt, nt);
        const int kb_lo = sp * nk_all / ns, kb_hi = (sp + 1) * nk_all / ns;
        for (int kb = kb_lo; kb < kb_hi; ++kb, ++it) {
          const uint32_t stage = it % NST, phase = (it / NST) & 1;
          const bool b_done = (int)it < pre;  // weight tile already requested above
          if (!b_done && !mbar_wait(&empty[stage], phase ^ 1)) {
            ok = false;
            break;
          }
          if (PAIR) {
            // the leader's barrier counts both CTAs' bytes; each CTA loads its own halves
            if (crank == 0 && !b_done) mbar_expect_tx(&full[stage], 2 * (A_BYTES + B_BYTES));
            const uint32_t fb = mapa_shared(smem_u32(&full[stage]), 0);
            tma_load_2d_pair(sA + stage * A_BYTES, &tmA, fb, kb * BK, (mt * 2 + (int)crank) * BM);
            if (!b_done)
              tma_load_2d_pair(sB + stage * B_BYTES, &tmB, fb, kb * BK, nt * BN + (int)crank * (BN / 2));
          } else {
            if (!b_done) mbar_expect_tx(&full[stage], A_BYTES + B_BYTES);
            tma_load_2d(sA + stage * A_BYTES, &tmA, &full[stage], kb * BK, mt * BM * MT);
            if (!b_done) tma_load_2d(sB + stage * B_BYTES, &tmB, &full[stage], kb * BK, nt * BN);
          }
        }
      }
    } else {
      pdl_wait();
    }
  } else if (warp == 1) {
    if (lane == 0 && crank == 0) {  // pair: the leader issues the MMAs for both CTAs
      constexpr uint32_t idesc = BF ? idesc_bf16(BN, PAIR ? 2 * BM : BM) : idesc_i8(BN, PAIR ? 2 * BM : BM);
      uint32_t it = 0, tile_i = 0;
      bool ok = true;
      for (int u = ustart; u < total && ok; u += ustride, ++tile_i) {
        const uint32_t buf = tile_i & 1, use = tile_i >> 1;
        int t_, sp, ns;
        unit_info(p, u, t_, sp, ns);
        const int kb_lo = sp * nk_all / ns, kb_hi = (sp + 1) * nk_all / ns;
        if (!mbar_wait(&tempty[buf], (use & 1) ^ 1)) break;
        fence_after();
        for (int kb = kb_lo; kb < kb_hi; ++kb, ++it) {
          const bool second = DUAL && kb >= p.ksplit;
          const uint32_t d_tmem = tmem_base + buf * ACC_COLS + (second ? BN : 0);
          const int kb0 = second ? kb - p.ksplit : kb - kb_lo;
          const uint32_t stage = it % NST, phase = (it / NST) & 1;
          if (!mbar_wait(&full[stage], phase)) {
            ok = false;
            break;
          }
          fence_after();
          const uint64_t adesc = smem_desc_sw128(sA + stage * A_BYTES);
          const uint64_t bdesc = smem_desc_sw128(sB + stage * B_BYTES);
#pragma unroll
          for (int kk = 0; kk < BK / 32; ++kk) {
            // advance 32 bytes along K inside the swizzle atom: +2 in 16-byte units
            if (PAIR) {
              if (BF)
                mma_bf16_pair(d_tmem, adesc + 2 * kk, bdesc + 2 * kk, idesc, (kb0 | kk) != 0);
              else
                mma_i8_pair(d_tmem, adesc + 2 * kk, bdesc + 2 * kk, idesc, (kb0 | kk) != 0);
            } else {
#pragma unroll
              for (int s = 0; s < MT; ++s)  // second M sub-tile: +16 KB = +1024 in 16-byte units
                if (BF)
                  mma_bf16(d_tmem + s * BN, adesc + 2 * kk + s * (BM * BK / 16), bdesc + 2 * kk, idesc,
                           (kb0 | kk) != 0);
                else
                  mma_i8(d_tmem + s * BN, adesc + 2 * kk + s * (BM * BK / 16), bdesc + 2 * kk, idesc,
                         (kb0 | kk) != 0);
            }
          }
          if (PAIR)
            mma_commit_pair(&empty[stage]);
          else
            mma_commit(&empty[stage]);
        }
        if (ok) {
          if (PAIR)
            mma_commit_pair(&tfull[buf]);
          else
            mma_commit(&tfull[buf]);
        }
      }
    }
  } else {
    // epilogue warps 2..9 -> TMEM lane quarter q = warp % 4
    const int q = warp & 3;
    const int half = (warp - 2) >> 2;  // which half of the tile's columns this warp stores
    uint32_t tile_i = 0;
    // DUAL with TMA: the local / gate operands do not depend on the accumulators, so each
    // chunk's tiles are requested one tile ahead, as soon as this tile's chunk has been read.
    const int ew = warp - 2;
    const bool dual_tma = DUAL && p.dual_tma;
    // A chunk's tiles are loaded (and its barrier completes a phase) only when the chunk has
    // columns below N and rows below M; the consumer tests the same condition and keeps its own
    // per-chunk phase bit, so skipped chunks never desynchronise the parity.
    auto issue_in = [&](int smt, int snt, int cc) {
      const int x = snt * BN + (half * DCH + cc) * 32;
      if (lane == 0 && x < p.N && smt * BM + q * 32 < p.M) {
        uint64_t *bar = &pbar[ew * DCH + cc];
        mbar_expect_tx(bar, 2 * 2048);
        uint8_t *dst = sP + (ew * DCH + cc) * 2 * 2048;
        tma_load_2d(dst, &tmL, bar, x, smt * BM + q * 32);
        tma_load_2d(dst + 2048, &tmG, bar, x, smt * BM + q * 32);
      }
    };
    // byte offset of 16-byte unit j of row r in a 32 x 64 B tile with the 64-byte swizzle
    auto sw64 = [](int r, int j) -> uint32_t { return (uint32_t)(r * 64 + ((j ^ ((r >> 1) & 3)) << 4)); };
    bool epi_ok = true;
    int nsplit = 0;  // split units this CTA's epilogue has handled (the same count in every warp)
    uint32_t in_phase = 0;  // bit cc: parity of chunk cc's next barrier phase
    // release of a TMEM buffer: to this CTA's barrier, or the pair leader's
    auto release = [&](uint32_t b) {
      if (lane != 0) return;
      if (PAIR)
        mbar_arrive_cluster(mapa_shared(smem_u32(&tempty[b]), 0));
      else
        mbar_arrive(&tempty[b]);
    };
    for (int u = ustart; u < total; u += ustride, ++tile_i) {
      int mt, nt, t_u, sp_u, ns_u;
      unit_info(p, u, t_u, sp_u, ns_u);
      tile_coords(p, t_u, mt, nt);
      const uint32_t buf = tile_i & 1, use = tile_i >> 1;
      if (dual_tma && tile_i == 0) {
#pragma unroll
        for (int cc = 0; cc < DCH; ++cc) issue_in(mt, nt, cc);
      }
      const int sub = MT == 2 ? half : 0;  // skinny tiles: each warp half owns one M sub-tile
      const int row = (PAIR ? mt * 2 + (int)crank : mt * MT + sub) * BM + q * 32 + lane;
      const bool row_ok = row < p.M;
      // dequantisation factors: loaded before the accumulator wait, so that their latency hides
      // behind this tile's MMAs (w4[i]: per-row factor of weight row n0 + lane of this warp's
      // i-th chunk; the SwiGLU tile uses gate rows in w4[0..1] and up rows in w4[2..3])
      const float xs = BF ? 1.f : (row_ok ? __ldg(p.inv_scale + row) : 0.f);
      const float wd0 = BF ? 1.f : __ldg(p.w_deq);
      float w4[4] = {0.f, 0.f, 0.f, 0.f};
      if (!BF && !DUAL && p.per_row) {
        if (BN == 256 && MT == 1 && p.swiglu) {
#pragma unroll
          for (int i = 0; i < 2; ++i) {
            const int ng = nt * BN + (half * 2 + i) * 32 + lane;
            if (ng < p.N) w4[i] = __ldg(p.w_deq + ng);
            if (ng + 128 < p.N) w4[2 + i] = __ldg(p.w_deq + ng + 128);
          }
        } else {
          const int c0 = MT == 2 ? 0 : half * (BN / 64);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int n = nt * BN + (c0 + i) * 32 + lane;
            if (i < (MT == 2 ? BN / 32 : BN / 64) && n < p.N) w4[i] = __ldg(p.w_deq + n);
          }
        }
      }
      if (!mbar_wait(&tfull[buf], use & 1)) break;
      if (p.pdl_late && warp == 2 && lane == 0 && u + ustride >= total) pdl_trigger();
      fence_after();
      // split-K: the other splits' partial sums of this tile are added to the accumulators read
      // from TMEM (only in the split that arrives last, see Params)
      bool fix = false;
      // A partial slice is stored in 32 x 32 blocks (32 rows of this warp, 32 columns), each
      // lane-major: int4 jj of lane l holds columns 4jj..4jj+3 of row l, so every warp-wide
      // access covers 512 contiguous bytes.
      const int rblk = (row - lane) >> 5;
      auto part_blk = [&](int slice, int n0) -> int4 * {
        return reinterpret_cast<int4 *>(p.part) +
               (((int64_t)slice * p.part_rb + rblk) * p.part_cb + (n0 >> 5)) * 256;
      };
      // the other splits' slices, two per round trip to L2
      auto acc_fix = [&](uint32_t (&r)[32], int n0) {
        if (!fix || n0 >= p.N) return;
        for (int k = 0; k < ns_u - 1; k += 2) {
          const int s_a = k < sp_u ? k : k + 1;
          const int s_b = k + 1 < sp_u ? k + 1 : k + 2;
          const bool two = k + 1 < ns_u - 1;
          const int4 *ba = part_blk(s_a, n0);
          const int4 *bb = part_blk(two ? s_b : s_a, n0);
          int4 va[8], vb[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) va[j] = __ldcg(ba + j * 32 + lane);
          if (two) {
#pragma unroll
            for (int j = 0; j < 8; ++j) vb[j] = __ldcg(bb + j * 32 + lane);
          } else {
#pragma unroll
            for (int j = 0; j < 8; ++j) vb[j] = make_int4(0, 0, 0, 0);
          }
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            r[4 * j] += (uint32_t)va[j].x + (uint32_t)vb[j].x;
            r[4 * j + 1] += (uint32_t)va[j].y + (uint32_t)vb[j].y;
            r[4 * j + 2] += (uint32_t)va[j].z + (uint32_t)vb[j].z;
            r[4 * j + 3] += (uint32_t)va[j].w + (uint32_t)vb[j].w;
          }
        }
      };
      // Store one 32 x 32 chunk (lane l holds row rbase + l) through the warp's staging block:
      // bf16 rows of 64 B go out 8 rows per instruction, fp32 rows of 128 B 4 rows per
      // instruction.  Warp-collective; rows >= M are skipped.  Full chunks only (n0 + 32 <= width).
      auto stage_store = [&](const float (&v)[32], int rbase, int n0) {
        const uint32_t st = smem_u32(sStage + ew * 4096);
        __syncwarp();  // the previous chunk's reads of the block are done
        if (p.out_dtype == TESM_BF16) {
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            __nv_bfloat162 h[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) h[e] = __floats2bfloat162_rn(v[8 * j + 2 * e], v[8 * j + 2 * e + 1]);
            const uint4 u4 = *reinterpret_cast<uint4 *>(h);
            asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};\n" ::"r"(st + lane * 64 + ((j ^ ((lane >> 1) & 3)) << 4)),
                         "r"(u4.x), "r"(u4.y), "r"(u4.z), "r"(u4.w));
          }
          __syncwarp();
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int rr = i * 8 + (lane >> 2), j = lane & 3;
            const uint4 u4 = lds128(st + rr * 64 + ((j ^ ((rr >> 1) & 3)) << 4));
            if (rbase + rr < p.M)
              *reinterpret_cast<uint4 *>(reinterpret_cast<__nv_bfloat16 *>(p.out) + (int64_t)(rbase + rr) * p.ldo +
                                         n0 + j * 8) = u4;
          }
        } else {
#pragma unroll
          for (int j = 0; j < 8; ++j)
            asm volatile("st.shared.v4.f32 [%0], {%1,%2,%3,%4};\n" ::"r"(st + lane * 128 + ((j ^ (lane & 7)) << 4)),
                         "f"(v[4 * j]), "f"(v[4 * j + 1]), "f"(v[4 * j + 2]), "f"(v[4 * j + 3]));
          __syncwarp();
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int rr = i * 4 + (lane >> 3), j = lane & 7;
            const uint4 u4 = lds128(st + rr * 128 + ((j ^ (rr & 7)) << 4));
            if (rbase + rr < p.M)
              *reinterpret_cast<uint4 *>(reinterpret_cast<float *>(p.out) + (int64_t)(rbase + rr) * p.ldo + n0 +
                                         j * 4) = u4;
          }
        }
      };
      if (!DUAL && ns_u > 1) {
        // split unit: every split finalises the 32-column chunks c with c % ns == its split
        // index (a reduce-scatter).  Phase 1 stores the chunks the other splits own into this
        // split's slice; after every split of the tile has stored (counted in cnt), each one adds
        // the others' slices to its own chunks and runs the epilogue on them.  All splits of a
        // tile run in the same round of the persistent loop, so the wait always ends.
        const int c_lo = MT == 2 ? 0 : half * (BN / 64), c_hi = MT == 2 ? BN / 32 : (half + 1) * (BN / 64);
#pragma unroll 1
        for (int c = c_lo; c < c_hi; ++c) {
          const int owner = (p.swiglu ? (c & 3) : c) % ns_u;
          if (owner == sp_u) continue;
          uint32_t r[32];
          tmem_ld32(tmem_base + ((uint32_t)(q * 32) << 16) + buf * ACC_COLS + sub * BN + c * 32, r);
          const int n0 = nt * BN + c * 32;
          if (n0 >= p.N) continue;
          int4 *blk = part_blk(sp_u, n0);  // rows past M and columns past N are stored too (unused)
#pragma unroll
          for (int j = 0; j < 8; ++j)
            __stcg(blk + j * 32 + lane, make_int4((int)r[4 * j], (int)r[4 * j + 1], (int)r[4 * j + 2],
                                                  (int)r[4 * j + 3]));
        }
        // Meeting.  Each epilogue warp publishes its partial stores to the CTA (release at CTA
        // scope on a shared word); warp 0 of the epilogue acquires all eight, counts the CTA in
        // the tile's counter with one release at GPU scope (cumulative over the stores it has
        // acquired), waits (bounded) until every split has counted, and hands the outcome to the
        // other warps through a second shared word.  Shared-memory words with bounded waits
        // instead of a named barrier: a warp that gave up on an earlier wait cannot leave the
        // others blocked.
        __syncwarp();
        ++nsplit;
        int ok = 0;
        if (lane == 0) red_release_cta(&s_arrive, 1);
        if (ew == 0 && lane == 0) {
          const long long t0 = clock64();
          bool met = true;
          while (ld_acquire_cta(&s_arrive) < EPI_WARPS * nsplit) {
            if (clock64() - t0 > kWaitCycles) {
              flag_timeout();
              met = false;
              break;
            }
          }
          if (met) {
            int *cn = p.cnt + (int64_t)t_u * 2 + (int)crank;
            red_release_gpu(cn, 1);
            const long long t1 = clock64();
            while (ld_acquire_gpu(cn) < ns_u) {  // every split of the tile has stored its partials
              if (clock64() - t1 > kWaitCycles) {
                flag_timeout();
                met = false;
                break;
              }
            }
            if (met) {
              ok = 1;
              // second count: the split that completes it resets the counter for the next call
              // (every split has passed the wait above by then)
              if (atomicAdd(cn, 1) == 2 * ns_u - 1) *cn = 0;
            }
          }
          s_last = ok;
          st_release_cta(&s_decided, nsplit);
        } else if (lane == 0) {
          const long long t0 = clock64();
          int d;
          while ((d = ld_acquire_cta(&s_decided)) < nsplit) {
            if (clock64() - t0 > kWaitCycles) {
              flag_timeout();
              break;
            }
          }
          ok = d >= nsplit ? *(volatile int *)&s_last : 0;
        }
        fix = __shfl_sync(0xffffffffu, ok, 0) != 0;
        if (!fix) {
          fence_before();
          __syncwarp();
          release(buf);
          continue;
        }
        __threadfence_block();
      }
      if (DUAL && dual_tma) {
        const float s1 = xs * wd0, s2 = (row_ok ? p.inv_scale2[row] : 0.f) * p.w_deq2[0];
        int mtn = 0, ntn = 0;
        const int un = u + ustride;
        if (un < total) {
          int tn, spn, nsn;
          unit_info(p, un, tn, spn, nsn);
          tile_coords(p, tn, mtn, ntn);
        }
#pragma unroll
        for (int cc = 0; cc < DCH; ++cc) {
          const int c = half * DCH + cc;
          const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + buf * ACC_COLS + c * 32;
          const int n0 = nt * BN + c * 32;
          uint32_t r[32];
          float v[32];
          tmem_ld32(tbase, r);  // acc1 (state_proj)
          uint4 pl[4], pg[4];
          const bool have = n0 < p.N && mt * BM + q * 32 < p.M;
          if (have) {
            if (!mbar_wait(&pbar[ew * DCH + cc], (in_phase >> cc) & 1)) epi_ok = false;
            in_phase ^= 1u << cc;
          }
          const uint32_t sin = smem_u32(sP + (ew * DCH + cc) * 2 * 2048);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            pl[j] = lds128(sin + sw64(lane, j));
            pg[j] = lds128(sin + 2048 + sw64(lane, j));
          }
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const __nv_bfloat162 *hl = reinterpret_cast<const __nv_bfloat162 *>(&pl[j]);
            const __nv_bfloat162 *hg = reinterpret_cast<const __nv_bfloat162 *>(&pg[j]);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float2 fl = __bfloat1622float2(hl[e]), fg = __bfloat1622float2(hg[e]);
              const int jj = 8 * j + 2 * e;
              v[jj] = combine_first(fl.x, fg.x, acc_to_f(r[jj]), s1);
              v[jj + 1] = combine_first(fl.y, fg.y, acc_to_f(r[jj + 1]), s1);
            }
          }
          // every lane has consumed its slot values (register dependencies above): refill the
          // chunk's slots with the next tile's tiles
          __syncwarp();
          if (un < total && epi_ok) issue_in(mtn, ntn, cc);
          tmem_ld32(tbase + BN, r);  // acc2 (ent_proj)
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = combine_second(v[j], acc_to_f(r[j]), s2);
          // the output slot of this chunk was last used DCH store groups ago
          if (lane == 0) bulk_wait_read<DCH - 1>();
          __syncwarp();
          uint8_t *so = sO + (ew * DCH + cc) * 2048;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            __nv_bfloat162 h[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) h[e] = __floats2bfloat162_rn(v[8 * j + 2 * e], v[8 * j + 2 * e + 1]);
            *reinterpret_cast<uint4 *>(so + sw64(lane, j)) = *reinterpret_cast<uint4 *>(h);
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            if (have) tma_store_2d(&tmO, so, n0, mt * BM + q * 32);  // rows >= M, cols >= N are clipped
            bulk_commit();
          }
        }
        fence_before();
        __syncwarp();
        release(buf);
        if (!epi_ok) break;
        continue;
      }
      if (DUAL) {
        const float xs2 = row_ok ? p.inv_scale2[row] : 0.f;
        const float s1 = xs * wd0, s2 = xs2 * p.w_deq2[0];
        const int esz = p.proj_dtype == TESM_BF16 ? 2 : 4;
        const uint8_t *prow = reinterpret_cast<const uint8_t *>(p.proj) + (int64_t)(row_ok ? row : 0) * p.ldp * esz;
#pragma unroll 1
        for (int c = half * DCH; c < (half + 1) * DCH; ++c) {
          const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + buf * ACC_COLS + c * 32;
          const int n0 = nt * BN + c * 32;
          const bool full = p.proj_vec && n0 + 32 <= p.N;
          float v[32];
          uint32_t r[32];
          tmem_ld32(tbase, r);
          {
            uint32_t r2[32];
            tmem_ld32(tbase + BN, r2);
            if (!row_ok || n0 >= p.N) continue;
            const uint32_t(&r1)[32] = r;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              float loc[16], gt[16];
              load16(prow + (int64_t)p.c_local * esz, p.proj_dtype, n0 + 16 * h, p.N, full, loc);
              load16(prow + (int64_t)p.c_gate * esz, p.proj_dtype, n0 + 16 * h, p.N, full, gt);
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                const int jj = 16 * h + j;
                v[jj] = combine_second(combine_first(loc[j], gt[j], acc_to_f(r1[jj]), s1), acc_to_f(r2[jj]), s2);
              }
            }
          }
          const bool vs = p.vec_store && n0 + 32 <= p.N;
          uint8_t *orow = reinterpret_cast<uint8_t *>(p.out) + (int64_t)row * p.ldo * (p.out_dtype == TESM_BF16 ? 2 : 4);
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            float w16[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) w16[j] = v[16 * h + j];
            store16(orow, p.out_dtype, n0 + 16 * h, p.N, vs, w16);
          }
        }
        fence_before();
        __syncwarp();
        release(buf);
        continue;
      }
      if (BN == 256 && MT == 1 && p.swiglu) {
        // columns [0,128) of the tile are gate rows, [128,256) the matching up rows
#pragma unroll 1
        for (int c = half * 2; c < half * 2 + 2; ++c) {
          uint32_t rg[32], ru[32];
          const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + buf * BN;
          if (fix && c % ns_u != sp_u) continue;  // split-K: another split finalises this chunk
          tmem_ld32(tbase + c * 32, rg);
          tmem_ld32(tbase + 128 + c * 32, ru);
          const int ng = nt * BN + c * 32;    // weight row of the first gate column
          const int no = nt * 128 + c * 32;   // output column
          if (ng >= p.N) continue;
          acc_fix(rg, ng);
          acc_fix(ru, ng + 128);
          float v[32];
          // per-row dequantisation factors of the chunk's 32 gate and 32 up rows: one coalesced
          // load each, handed to the lanes by shuffles
          // (the conversion and transcendental unit is the epilogue's bottleneck: accumulators
          // are converted with integer adds when |acc| < 2^22, and silu takes one exp2 and one
          // reciprocal, relative error a few ulp)
          const float dg = (c & 1) ? w4[1] : w4[0], du = (c & 1) ? w4[3] : w4[2];
          const bool small_acc = p.K < 32768;  // |acc| <= 128 K < 2^22
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const float ag = small_acc ? acc_to_f(rg[j]) : (float)(int32_t)rg[j];
            const float au = small_acc ? acc_to_f(ru[j]) : (float)(int32_t)ru[j];
            const float g = ag * xs * __shfl_sync(0xffffffffu, dg, j);
            const float u = au * xs * __shfl_sync(0xffffffffu, du, j);
            v[j] = __fdividef(g, 1.f + __expf(-g)) * u;
          }
          const int nout = p.N / 2;
          if (p.vec_store && no + 32 <= nout) {
            stage_store(v, row - lane, no);
            continue;
          }
          if (!row_ok) continue;
          for (int j = 0; j < 32; ++j)
            if (no + j < nout) store_f(p.out, p.out_dtype, (int64_t)row * p.ldo + no + j, v[j]);
        }
        fence_before();
        __syncwarp();
        release(buf);
        continue;
      }
      const int c_lo = MT == 2 ? 0 : half * (BN / 64), c_hi = MT == 2 ? BN / 32 : (half + 1) * (BN / 64);
#pragma unroll 1
      for (int c = c_lo; c < c_hi; ++c) {
        if (fix && c % ns_u != sp_u) continue;  // split-K: another split finalises this chunk
        uint32_t r[32];
        const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + buf * ACC_COLS + sub * BN + c * 32;
        tmem_ld32(taddr, r);
        const int n0 = nt * BN + c * 32;
        if (n0 >= p.N) continue;
        acc_fix(r, n0);
        float v[32];
        const int ci = c - c_lo;
        const float wdl = p.per_row ? (ci == 0 ? w4[0] : ci == 1 ? w4[1] : ci == 2 ? w4[2] : w4[3]) : wd0;
        const bool small_acc = p.K < 32768;  // |acc| <= 128 K < 2^22: convert without the XU pipe
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const float wd = p.per_row ? __shfl_sync(0xffffffffu, wdl, j) : wd0;
          v[j] = BF ? __uint_as_float(r[j]) : (small_acc ? acc_to_f(r[j]) : (float)(int32_t)r[j]) * xs * wd;
        }
        if (p.out && p.vec_store && n0 + 32 <= p.N && !p.acc_out) {
          stage_store(v, row - lane, n0);
          continue;
        }
        if (!row_ok) continue;
        if (p.acc_out) {
          int32_t *arow = p.acc_out + (int64_t)row * p.ld_acc;
          for (int j = 0; j < 32; ++j)
            if (n0 + j < p.N) arow[n0 + j] = (int32_t)r[j];
        }
        if (!p.out) continue;  // accumulator-only call (tensor-parallel partial sums)
        if (p.vec_store && n0 + 32 <= p.N) {
          if (p.out_dtype == TESM_BF16) {
            uint4 *dst = reinterpret_cast<uint4 *>(reinterpret_cast<__nv_bfloat16 *>(p.out) + (int64_t)row * p.ldo + n0);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              __nv_bfloat162 h[4];
#pragma unroll
              for (int e = 0; e < 4; ++e) h[e] = __floats2bfloat162_rn(v[8 * j + 2 * e], v[8 * j + 2 * e + 1]);
              dst[j] = *reinterpret_cast<uint4 *>(h);
            }
          } else {
            float4 *dst = reinterpret_cast<float4 *>(reinterpret_cast<float *>(p.out) + (int64_t)row * p.ldo + n0);
#pragma unroll
            for (int j = 0; j < 8; ++j) dst[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
          }
        } else {
          for (int j = 0; j < 32; ++j)
            if (n0 + j < p.N) store_f(p.out, p.out_dtype, (int64_t)row * p.ldo + n0 + j, v[j]);
        }
      }
      fence_before();
      __syncwarp();
      release(buf);
    }
    // TMA stores still reading this warp's output slots must finish before the CTA exits
    if (dual_tma && lane == 0) bulk_wait_all();
  }

  fence_before();
  if (PAIR)
    cluster_sync();  // the leader's MMAs into this CTA's TMEM are complete
  else
    __syncthreads();
  if (warp == 1) {
    fence_after();
    if (PAIR)
      asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;\n" ::"r"(tmem_base), "r"(TMEM_COLS));
    else
      asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem_base), "r"(TMEM_COLS));
  }
}

// Split-K finalize: sum the per-split int32 partials, scale (optionally apply the SiLU gate over
// 128-row interleaved gate/up blocks) and write the output.
__global__ void k_splitk_finalize(const int32_t *ws, int splits, int M, int N, const float *inv_scale,
                                  const float *w_deq, int per_row, int swiglu, void *out, int out_dtype, int64_t ldo,
                                  int32_t *acc_out, int64_t ld_acc) {
  pdl_trigger();
  pdl_wait();
  const int nout = swiglu ? N / 2 : N;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)M * nout) return;
  const int m = (int)(i / nout), n = (int)(i - (int64_t)m * nout);
  const float xs = inv_scale[m];
  const int64_t slice = (int64_t)M * N;
  if (swiglu) {
    const int b = n >> 7, j = n & 127;
    const int ng = b * 256 + j, nu = ng + 128;
    int32_t ag = 0, au = 0;
    for (int s = 0; s < splits; ++s) {
      ag += ws[s * slice + (int64_t)m * N + ng];
      au += ws[s * slice + (int64_t)m * N + nu];
    }
    const float g = (float)ag * xs * w_deq[ng];
    const float u = (float)au * xs * w_deq[nu];
    store_f(out, out_dtype, (int64_t)m * ldo + n, (g / (1.f + expf(-g))) * u);
  } else {
    int32_t a = 0;
    for (int s = 0; s < splits; ++s) a += ws[s * slice + (int64_t)m * N + n];
    const float wd = per_row ? w_deq[n] : w_deq[0];
    if (out) store_f(out, out_dtype, (int64_t)m * ldo + n, (float)a * xs * wd);
    if (acc_out) acc_out[(int64_t)m * ld_acc + n] = a;
  }
}

// The dual-accumulator combine epilogue on int32 accumulators summed elsewhere (tensor-parallel
// row splits of state_proj / ent_proj): out = local + sigmoid(gate) * acc1 * (inv1 * deq1)
// + acc2 * (inv2 * deq2), the arithmetic of the GEMM's epilogue.
__global__ void k_combine_acc(const int32_t *acc1, const int32_t *acc2, int64_t lda, int M, int N,
                              const float *inv1, const float *inv2, const float *deq1, const float *deq2,
                              const void *proj, int proj_dtype, int64_t ldp, int c_local, int c_gate, void *out,
                              int out_dtype, int64_t ldo) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)M * N) return;
  const int m = (int)(i / N), n = (int)(i - (int64_t)m * N);
  const float s1 = inv1[m] * deq1[0], s2 = inv2[m] * deq2[0];
  const float loc = load_f(proj, proj_dtype, (int64_t)m * ldp + c_local + n);
  const float gate = load_f(proj, proj_dtype, (int64_t)m * ldp + c_gate + n);
  const float v = combine_second(combine_first(loc, gate, acc_to_f((uint32_t)acc1[(int64_t)m * lda + n]), s1),
                                 acc_to_f((uint32_t)acc2[(int64_t)m * lda + n]), s2);
  store_f(out, out_dtype, (int64_t)m * ldo + n, v);
}

// ------------------------------------------------------------ host side
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

// 2-D uint8 tensor map: inner dim `inner` bytes, `outer` rows, row pitch `ld` bytes.
static int make_map(CUtensorMap *map, const void *ptr, int64_t inner, int64_t outer, int64_t ld, int box_outer) {
  auto fn = encode_fn();
  if (!fn) return fail(TESM_ELAUNCH, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
  cuuint64_t strides[1] = {(cuuint64_t)ld};
  cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(ptr), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(TESM_EINVAL, "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
  return TESM_OK;
}

// bf16 matrix (inner columns, outer rows, row pitch ld elements) in 32 x 32 boxes with the
// 64-byte swizzle: the combine epilogue's local / gate / output tiles.
static int make_map_bf16_32(CUtensorMap *map, const void *ptr, int64_t inner, int64_t outer, int64_t ld) {
  auto fn = encode_fn();
  if (!fn) return fail(TESM_ELAUNCH, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(ptr), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(TESM_EINVAL, "cuTensorMapEncodeTiled (bf16) failed (" + std::to_string((int)r) + ")");
  return TESM_OK;
}

template <int BN, bool DUAL = false, int MT = 1, bool PAIR = false, bool BF = false>
static int launch(const int8_t *A, int64_t lda, const int8_t *B, int64_t ldb, Params p, cudaStream_t st) {
  CUtensorMap ma, mb, ml, mg, mo;
  int rc = make_map(&ma, A, p.K, p.M, lda, BM * MT);
  if (rc) return rc;
  static const int pdl_late_env = [] {
    const char *e = getenv("TESM_PDL_GEMM_LATE");
    return e ? atoi(e) : 1;
  }();
  p.pdl_late = pdl_late_env;
  rc = make_map(&mb, B, p.K, p.N, ldb, PAIR ? BN / 2 : BN);
  if (rc) return rc;
  ml = mg = mo = ma;  // unused unless dual_tma
  if (DUAL && p.dual_tma) {
    const __nv_bfloat16 *pr = reinterpret_cast<const __nv_bfloat16 *>(p.proj);
    if ((rc = make_map_bf16_32(&ml, pr + p.c_local, p.N, p.M, p.ldp))) return rc;
    if ((rc = make_map_bf16_32(&mg, pr + p.c_gate, p.N, p.M, p.ldp))) return rc;
    if ((rc = make_map_bf16_32(&mo, p.out, p.N, p.M, p.ldo))) return rc;
  }
  constexpr int NST = PAIR ? 6 : STAGES;
  const size_t smem = 1024 + (size_t)NST * (MT * BM * BK + (PAIR ? BN / 2 : BN) * BK) +
                      (DUAL ? 1024 + (size_t)EPI_WARPS * (BN / 64) * 3 * 2048 : 1024 + (size_t)EPI_WARPS * 4096);
  auto kern = k_gemm_i8<BN, DUAL, MT, PAIR, BF>;
  static bool attr = false;
  static int max_clusters = 0;
  if (!attr) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    attr = true;
  }
  p.num_m_tiles = (int)ceil_div(p.M, BM * MT * (PAIR ? 2 : 1));
  p.num_n_tiles = (int)ceil_div(p.N, BN);
  p.num_k_blocks = (int)ceil_div(p.K, BK);
  static const int gm_force = [] {
    const char *e = getenv("TESM_GEMM_GROUP_M");  // tuning override: m-tiles per raster group
    return e ? atoi(e) : 0;
  }();
  // CTA pairs: 32 m-tiles per raster group for wide, short-K weights (in_proj, gate/up: the
  // weight is swept once per group, so fewer groups halve its re-reads), 8 otherwise (ncu at
  // M = 131072: DRAM bytes 4.57 -> 4.18 GB in_proj, 11.55 -> 5.86 GB gate/up)
  p.group_m = gm_force > 0 ? gm_force : (PAIR ? (p.N >= 8192 && p.K <= 4096 ? 32 : 8) : 16);
  const int tiles = p.num_m_tiles * p.num_n_tiles;
  if (PAIR && !max_clusters) {
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = 2;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.blockDim = dim3(NUM_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    cfg.gridDim = dim3(2 * (sm_count() / 2));
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      n = sm_count() / 2;
    }
    max_clusters = n;
  }
  // split-K when the tiles do not fill the machine (small M): whole tiles first, the tail (or,
  // with fewer tiles than workers, every tile) cut into k-ranges so the units fill the workers
  p.splits = 1;
  p.n_full = tiles;
  const int workers = PAIR ? max_clusters : sm_count();
  if (!BF && !DUAL && MT == 1 && p.ws && p.ws_bytes > (int64_t)kCounterInts * 4 && p.num_k_blocks >= 4 &&
      tiles * 2 <= kCounterInts) {
    const int nfull = tiles >= workers ? (tiles / workers) * workers : 0;
    const int rem = tiles - nfull;
    static const int smax = [] {
      const char *e = getenv("TESM_SPLITK_MAX");  // tuning override: most splits per tile
      return e ? atoi(e) : 8;
    }();
    if (rem > 0) {
      int s = workers / rem;
      if (s > smax) s = smax;
      if (s > BN / 32 / (p.swiglu ? 2 : 1)) s = BN / 32 / (p.swiglu ? 2 : 1);  // chunks a split owns
      if (s > p.num_k_blocks / 2) s = p.num_k_blocks / 2;
      p.part_rb = p.num_m_tiles * (BM * MT * (PAIR ? 2 : 1)) / 32;
      p.part_cb = (int)ceil_div(p.N, 32);
      const int64_t slice = (int64_t)p.part_rb * 32 * p.part_cb * 32 * 4;
      while (s >= 2 && s * slice > p.ws_bytes - (int64_t)kCounterInts * 4) --s;
      if (s >= 2) {
        p.splits = s;
        p.n_full = nfull;
        p.cnt = p.ws;
        p.part = p.ws + kCounterInts;
      }
    }
  }
  const int total = p.n_full + (tiles - p.n_full) * p.splits;
  if (PAIR) {
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute at[2];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = 2;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.blockDim = dim3(NUM_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cfg.attrs = at;
    cfg.numAttrs = pdl_enabled() ? 2 : 1;
    const int clusters = total < max_clusters ? total : max_clusters;
    cfg.gridDim = dim3(2 * clusters);
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, ma, mb, ml, mg, mo, p);
    if (e != cudaSuccess) return fail(TESM_ELAUNCH, std::string("gemm_i8 (CTA pairs): ") + cudaGetErrorString(e));
    return check_launch("gemm_i8 (CTA pairs)");
  }
  const int grid = total < sm_count() ? total : sm_count();
  return launch_k("gemm_i8", kern, dim3(grid), dim3(NUM_THREADS), smem, st, ma, mb, ml, mg, mo, p);
}

// CTA pairs for large plain / SwiGLU GEMMs: enough 256 x 256 tiles to fill every SM pair.
// TESM_GEMM_PAIR=0 / 1 forces the choice (tuning and tests).
static bool use_pairs(int64_t M, int64_t N) {
  static int force = -2;
  if (force == -2) {
    const char *e = getenv("TESM_GEMM_PAIR");
    force = e ? atoi(e) : -1;
  }
  if (force >= 0) return force > 0;
  return ceil_div(M, 256) * ceil_div(N, 256) >= 2 * (sm_count() / 2);
}

}  // namespace tc
}  // namespace tesm

using namespace tesm;

extern "C" int tesm_b200_gemm_i8_swiglu(const int8_t *codes, int64_t ld_codes, const float *inv_scale,
                                        const int8_t *tern, int64_t ld_tern, const float *w_deq, int64_t M, int64_t F,
                                        int64_t K, void *out, int out_dtype, int64_t ldo, int32_t *splitk_ws,
                                        int64_t ws_bytes, tesm_stream_t stream) {
  if (M == 0) return TESM_OK;  // empty batch: nothing to do (its buffers may be null)
  TESM_REQUIRE(codes && inv_scale && tern && w_deq && out, "gemm_i8_swiglu: null pointer");
  TESM_REQUIRE(M >= 0 && F > 0 && F % 128 == 0 && K > 0 && M < (1ll << 31), "gemm_i8_swiglu: need F % 128 == 0");
  if (out_dtype != TESM_F32 && out_dtype != TESM_BF16) return fail(TESM_EDTYPE, "gemm_i8_swiglu: out dtype");
  TESM_REQUIRE(ld_codes >= K && ld_codes % 16 == 0 && ((uintptr_t)codes & 15) == 0, "gemm_i8_swiglu: codes layout");
  TESM_REQUIRE(ld_tern >= K && ld_tern % 16 == 0 && ((uintptr_t)tern & 15) == 0, "gemm_i8_swiglu: tern layout");
  TESM_REQUIRE(ldo >= F, "gemm_i8_swiglu: ldo < F");
  tc::Params p = {};
  p.inv_scale = inv_scale;
  p.w_deq = w_deq;
  p.per_row = 1;
  p.M = (int)M;
  p.N = (int)(2 * F);
  p.K = (int)K;
  p.out = out;
  p.out_dtype = out_dtype;
  p.ldo = ldo;
  p.swiglu = 1;
  if (splitk_ws && ((uintptr_t)splitk_ws & 15) == 0) {
    p.ws = splitk_ws;
    p.ws_bytes = ws_bytes;
  }
  const int esz = out_dtype == TESM_BF16 ? 2 : 4;
  p.vec_store = ((uintptr_t)out % 16 == 0) && ((ldo * esz) % 16 == 0);
  // CTA pairs when the 256 x 256 tiles fill the SM pairs, and for decode batches (129..256 rows,
  // where split-K fills them)
  if (tc::use_pairs(M, 2 * F) || (M > 128 && M <= 256 && p.ws))
    return tc::launch<256, false, 1, true>(codes, ld_codes, tern, ld_tern, p, (cudaStream_t)stream);
  return tc::launch<256>(codes, ld_codes, tern, ld_tern, p, (cudaStream_t)stream);
}

extern "C" int tesm_b200_gemm_i8_combine(const int8_t *codes, int64_t ld_codes, int64_t Kh, const float *inv1,
                                         const float *inv2, const int8_t *tern, int64_t ld_tern, const float *deq1,
                                         const float *deq2, const void *proj, int proj_dtype, int64_t ldp,
                                         int64_t c_local, int64_t c_gate, int64_t M, int64_t N, void *out,
                                         int out_dtype, int64_t ldo, tesm_stream_t stream) {
  if (M == 0) return TESM_OK;  // empty batch: nothing to do (its buffers may be null)
  TESM_REQUIRE(codes && inv1 && inv2 && tern && deq1 && deq2 && proj && out, "gemm_i8_combine: null pointer");
  TESM_REQUIRE(M >= 0 && N > 0 && Kh > 0 && Kh % 128 == 0 && M < (1ll << 31), "gemm_i8_combine: need Kh % 128 == 0");
  TESM_REQUIRE(Kh <= 16384, "gemm_i8_combine: d_state above 16384");
  if (out_dtype != TESM_F32 && out_dtype != TESM_BF16) return fail(TESM_EDTYPE, "gemm_i8_combine: out dtype");
  if (proj_dtype != TESM_F32 && proj_dtype != TESM_BF16) return fail(TESM_EDTYPE, "gemm_i8_combine: proj dtype");
  TESM_REQUIRE(ld_codes >= 2 * Kh && ld_codes % 16 == 0 && ((uintptr_t)codes & 15) == 0, "gemm_i8_combine: codes");
  TESM_REQUIRE(ld_tern >= 2 * Kh && ld_tern % 16 == 0 && ((uintptr_t)tern & 15) == 0, "gemm_i8_combine: tern");
  TESM_REQUIRE(ldo >= N && ldp >= c_local + N && ldp >= c_gate + N, "gemm_i8_combine: strides");
  tc::Params p = {};
  p.inv_scale = inv1;
  p.w_deq = deq1;
  p.inv_scale2 = inv2;
  p.w_deq2 = deq2;
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)(2 * Kh);
  p.ksplit = (int)(Kh / 128);
  p.out = out;
  p.out_dtype = out_dtype;
  p.ldo = ldo;
  p.proj = proj;
  p.proj_dtype = proj_dtype;
  p.ldp = ldp;
  p.c_local = (int)c_local;
  p.c_gate = (int)c_gate;
  const int esz = out_dtype == TESM_BF16 ? 2 : 4, psz = proj_dtype == TESM_BF16 ? 2 : 4;
  p.vec_store = ((uintptr_t)out % 16 == 0) && ((ldo * esz) % 16 == 0);
  p.proj_vec = ((uintptr_t)proj % 16 == 0) && ((ldp * psz) % 16 == 0) && ((c_local * psz) % 16 == 0) &&
               ((c_gate * psz) % 16 == 0);
  p.dual_tma = p.proj_vec && p.vec_store && proj_dtype == TESM_BF16 && out_dtype == TESM_BF16;
  // decode batches: 64-column tiles double the CTAs when 128-column tiles leave SMs idle
  static const int narrow = [] {
    const char *e = getenv("TESM_COMBINE_NARROW");  // tuning override: 0 = always 128 columns
    return e ? atoi(e) : 1;
  }();
  if (narrow && ceil_div(M, 128) * ceil_div(N, 128) < sm_count())
    return tc::launch<64, true>(codes, ld_codes, tern, ld_tern, p, (cudaStream_t)stream);
  return tc::launch<128, true>(codes, ld_codes, tern, ld_tern, p, (cudaStream_t)stream);
}

extern "C" int tesm_b200_gemm_i8(const int8_t *codes, int64_t ld_codes, const float *inv_scale, const int8_t *tern,
                                 int64_t ld_tern, const float *w_deq, int per_row, int64_t M, int64_t N, int64_t K,
                                 void *out, int out_dtype, int64_t ldo, int32_t *acc_out, int64_t ld_acc,
                                 int32_t *splitk_ws, int64_t ws_bytes, tesm_stream_t stream) {
  if (M == 0) return TESM_OK;  // empty batch: nothing to do (its buffers may be null)
  TESM_REQUIRE(codes && inv_scale && tern && w_deq && (out || acc_out), "gemm_i8: null pointer");
  TESM_REQUIRE(M > 0 && N > 0 && K > 0 && M < (1ll << 31) && N < (1ll << 31), "gemm_i8: bad shape");
  if (out_dtype != TESM_F32 && out_dtype != TESM_BF16) return fail(TESM_EDTYPE, "gemm_i8: out dtype");
  TESM_REQUIRE(ld_codes >= K && ld_codes % 16 == 0 && ((uintptr_t)codes & 15) == 0,
               "gemm_i8: codes rows must be 16-byte aligned with ld_codes >= K");
  TESM_REQUIRE(ld_tern >= K && ld_tern % 16 == 0 && ((uintptr_t)tern & 15) == 0,
               "gemm_i8: tern rows must be 16-byte aligned with ld_tern >= K");
  TESM_REQUIRE(ldo >= N, "gemm_i8: ldo < N");
  tc::Params p = {};
  p.inv_scale = inv_scale;
  p.w_deq = w_deq;
  p.per_row = per_row;
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.out = out;
  p.out_dtype = out_dtype;
  p.ldo = ldo;
  p.acc_out = acc_out;
  p.ld_acc = ld_acc;
  if (splitk_ws && ((uintptr_t)splitk_ws & 15) == 0) {
    p.ws = splitk_ws;
    p.ws_bytes = ws_bytes;
  }
  const int esz = out_dtype == TESM_BF16 ? 2 : 4;
  p.vec_store = ((uintptr_t)out % 16 == 0) && ((ldo * esz) % 16 == 0);
  cudaStream_t st = (cudaStream_t)stream;
  if (M <= 256) {  // decode-sized batches: narrow tiles, enough CTAs, weights streamed once
    static const int forced = [] {
      const char *e = getenv("TESM_SKINNY_BN");  // tuning override: 32, 64 or 128
      return e ? atoi(e) : 0;
    }();
    // CTA pairs (M = 256 MMAs, cta_group::2): each CTA stages only its 128 activation rows and
    // half of the weight tile, so per-CTA bytes per k-block halve and twice as many SMs work
    // (TESM_SKINNY_PAIR=0 selects the single-CTA skinny tiles below for every M)
    static const int pair = [] {
      const char *e = getenv("TESM_SKINNY_PAIR");
      return e ? atoi(e) : 1;
    }();
    // up to 128 rows leave half of each pair tile empty: pairs still win when N is small (fewer,
    // longer-K tiles: 4096 x 11008 at M = 128, 34.5 vs 43.7 us) but not for wide N
    // (11008 x 4096: 29.3 vs 24.8 us)
    // 129..256 rows: 256 x 256 pair tiles (the activation block is re-read once per 256 output
    // columns instead of once per 64 / 128) with split-K filling the SM pairs
    // (TESM_SKINNY_WIDE=0 selects the narrow pair tiles below)
    static const int wide = [] {
      const char *e = getenv("TESM_SKINNY_WIDE");
      return e ? atoi(e) : 1;
    }();
    if (pair && forced == 0 && wide && M > 128 && p.ws)
      return tc::launch<256, false, 1, true>(codes, ld_codes, tern, ld_tern, p, st);
    if (pair && forced == 0 && (M > 128 || N < 8192)) {
      if (N >= 8192) return tc::launch<128, false, 1, true>(codes, ld_codes, tern, ld_tern, p, st);
      return tc::launch<64, false, 1, true>(codes, ld_codes, tern, ld_tern, p, st);
    }
    if (forced == 128) return tc::launch<128, false, 2>(codes, ld_codes, tern, ld_tern, p, st);
    if (forced == 64) return tc::launch<64, false, 2>(codes, ld_codes, tern, ld_tern, p, st);
    if (forced == 32) return tc::launch<32, false, 2>(codes, ld_codes, tern, ld_tern, p, st);
    // every CTA re-reads the 256-row activation tile from L2, so wider N tiles cut L2 traffic;
    // narrower ones keep enough CTAs in flight when N is small
    // wide tiles cut the activation re-reads for large N; narrower ones keep CTAs in flight
    if (N >= 8192) return tc::launch<128, false, 2>(codes, ld_codes, tern, ld_tern, p, st);
    if (N >= 2048) return tc::launch<64, false, 2>(codes, ld_codes, tern, ld_tern, p, st);
    return tc::launch<32, false, 2>(codes, ld_codes, tern, ld_tern, p, st);
  }
  if (N <= 128) return tc::launch<128>(codes, ld_codes, tern, ld_tern, p, st);
  if (tc::use_pairs(M, N)) return tc::launch<256, false, 1, true>(codes, ld_codes, tern, ld_tern, p, st);
  return tc::launch<256>(codes, ld_codes, tern, ld_tern, p, st);
}

extern "C" int tesm_b200_acc_scale(const int32_t *acc, int64_t M, int64_t N, const float *inv_scale,
                                   const float *w_deq, int per_row, void *out, int out_dtype, int64_t ldo,
                                   tesm_stream_t stream) {
  if (M == 0) return TESM_OK;  // empty batch: nothing to do (its buffers may be null)
  TESM_REQUIRE(acc && inv_scale && w_deq && out, "acc_scale: null pointer");
  TESM_REQUIRE(M >= 0 && N > 0 && ldo >= N && M * N < (1ll << 40), "acc_scale: bad shape");
  if (out_dtype != TESM_F32 && out_dtype != TESM_BF16) return fail(TESM_EDTYPE, "acc_scale: out dtype");
  const int64_t n = M * N;
  tc::k_splitk_finalize<<<(unsigned)ceil_div(n, 256), 256, 0, (cudaStream_t)stream>>>(
      acc, 1, (int)M, (int)N, inv_scale, w_deq, per_row, 0, out, out_dtype, ldo, nullptr, 0);
  return check_launch("acc_scale");
}

extern "C" int tesm_b200_gemm_bf16(const void *a, int64_t lda, const void *b, int64_t ldb, int64_t M, int64_t N,
                                   int64_t K, void *out, int out_dtype, int64_t ldo, tesm_stream_t stream) {
  if (M == 0) return TESM_OK;
  TESM_REQUIRE(a && b && out, "gemm_bf16: null pointer");
  TESM_REQUIRE(M > 0 && N > 0 && K > 0 && M < (1ll << 31) && N < (1ll << 31), "gemm_bf16: bad shape");
  if (out_dtype != TESM_F32 && out_dtype != TESM_BF16) return fail(TESM_EDTYPE, "gemm_bf16: out dtype");
  TESM_REQUIRE(lda >= K && (lda * 2) % 16 == 0 && ((uintptr_t)a & 15) == 0, "gemm_bf16: A rows must be 16-byte aligned");
  TESM_REQUIRE(ldb >= K && (ldb * 2) % 16 == 0 && ((uintptr_t)b & 15) == 0, "gemm_bf16: B rows must be 16-byte aligned");
  TESM_REQUIRE(ldo >= N, "gemm_bf16: ldo < N");
  tc::Params p = {};
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)(K * 2);  // bytes: the operand tiles are moved and described as bytes
  p.out = out;
  p.out_dtype = out_dtype;
  p.ldo = ldo;
  const int esz = out_dtype == TESM_BF16 ? 2 : 4;
  p.vec_store = ((uintptr_t)out % 16 == 0) && ((ldo * esz) % 16 == 0);
  const int8_t *A = reinterpret_cast<const int8_t *>(a), *B = reinterpret_cast<const int8_t *>(b);
  cudaStream_t st = (cudaStream_t)stream;
  if (M > 128)  // 256-row tiles on CTA pairs
    return tc::launch<256, false, 1, true, true>(A, lda * 2, B, ldb * 2, p, st);
  return tc::launch<256, false, 1, false, true>(A, lda * 2, B, ldb * 2, p, st);
}

extern "C" int tesm_b200_combine_acc(const int32_t *acc1, const int32_t *acc2, int64_t ld_acc, int64_t M, int64_t N,
                                     const float *inv1, const float *inv2, const float *deq1, const float *deq2,
                                     const void *proj, int proj_dtype, int64_t ldp, int64_t c_local, int64_t c_gate,
                                     void *out, int out_dtype, int64_t ldo, tesm_stream_t stream) {
  if (M == 0) return TESM_OK;
  TESM_REQUIRE(acc1 && acc2 && inv1 && inv2 && deq1 && deq2 && proj && out, "combine_acc: null pointer");
  TESM_REQUIRE(M > 0 && N > 0 && ld_acc >= N && ldo >= N && M * N < (1ll << 40), "combine_acc: bad shape");
  if (proj_dtype != TESM_F32 && proj_dtype != TESM_BF16) return fail(TESM_EDTYPE, "combine_acc: proj dtype");
  if (out_dtype != TESM_F32 && out_dtype != TESM_BF16) return fail(TESM_EDTYPE, "combine_acc: out dtype");
  const int64_t n = M * N;
  tc::k_combine_acc<<<(unsigned)ceil_div(n, 256), 256, 0, (cudaStream_t)stream>>>(
      acc1, acc2, ld_acc, (int)M, (int)N, inv1, inv2, deq1, deq2, proj, proj_dtype, ldp, (int)c_local, (int)c_gate,
      out, out_dtype, ldo);
  return check_launch("combine_acc");
}
