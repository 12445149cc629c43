// pa_prefill_umma2.cu — multi-query attention over paged KV on pairs of SMs:
// 5th-generation tensor-core MMAs with cta_group::2 (M = 256 per instruction),
// fp16 / bf16, head_dim 128, sm_100a.
//
// Same contract, row layout and numerics as pa_prefill_umma.cu (the one-SM
// kernel this replaces for head_dim 128): rows of one KV head are token-major,
// query token t attends positions 0 .. L - q_len + t, fp32 scores, an online
// softmax per row with a lazily moved reference max, P applied as bf16 hi + lo.
// What changes is how the tensor cores are driven:
//
//  * Two CTAs on a pair of SMs (a cluster of 2) own 512 rows of one (sequence,
//    kv head): CTA c holds rows c*256 .. c*256+255 as two 128-row tiles, tile t
//    of the pair being CTA 0's tile t over CTA 1's tile t.  One thread of CTA 0
//    issues every MMA for the pair: S_t = Q_t K^T (M = 256, N = 64, K = 128)
//    and O_t += P_t V (M = 256, N = 128, K = 64).  Each MMA instruction does
//    twice the work of the one-SM kernel's (M = 128), so the pair issues half
//    as many per FLOP -- the issuing thread's ~50 cycles per instruction bound
//    the one-SM kernel (see pa_prefill_umma.cu).
//  * The B operand is split between the pair: for S each CTA holds 32 of the
//    chunk's 64 tokens of K, for O each CTA holds one 64-column half of V.  So
//    each CTA loads half of every K/V chunk (16 KB instead of 32), and twice
//    as many chunks fit its shared memory.  Each CTA's TMA loads signal CTA
//    0's full barrier (cta_group::2 form); CTA 0's commits signal both CTAs'
//    barriers (multicast); CTA 1's softmax warps arrive on CTA 0's barriers
//    (mapa + a cluster-scope release).  Loads never multicast.
//  * Each CTA's TMEM holds its own rows: S/P and O of its two tiles, as in the
//    one-SM kernel.
//
// Every wait is bounded; both CTAs meet at a cluster barrier before TMEM is
// released, so neither leaves while the other's MMAs may still run.
#include <math.h>

#include "pa_common.cuh"
#include "pa_internal.h"
#include "pa_tile_math.cuh"

namespace pa {

namespace {

constexpr int D2 = 128;                       // head_dim of this kernel
constexpr int kChunk2 = kUmmaChunkTokens;     // 64 tokens per chunk
constexpr int kStages2 = 8;                   // K/V chunks in flight per CTA
constexpr uint32_t kTmemCols2 = 512;          // per tile: S/P buffers (2 x 64) + O (128), at column 256 * tile
constexpr float kRescaleThreshold2 = 8.f;     // log2 units, as in the one-SM kernel
constexpr uint32_t K_HALF_BYTES = 32 * 128;   // 32 tokens x 64 dims x 2 B (one 128-byte swizzle atom column)
constexpr uint32_t K_BYTES = 2 * K_HALF_BYTES;            // this CTA's 32 tokens, both 64-dim halves
constexpr uint32_t V_BYTES = kChunk2 * 128;                // 64 tokens x this CTA's 64-dim half
constexpr uint32_t STAGE_BYTES2 = K_BYTES + V_BYTES;       // 16 KB
constexpr uint32_t QT_BYTES2 = 2 * 128 * 128;              // one 128-row tile of Q, both halves

template <typename T>
struct kFmt2;
template <>
struct kFmt2<__half> {
  static constexpr uint32_t value = 0;
};
template <>
struct kFmt2<__nv_bfloat16> {
  static constexpr uint32_t value = 1;
};

__device__ __forceinline__ uint64_t desc_sw128(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((addr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;  // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;  // 128-byte swizzle
  return d;
}

// kind::f16 instruction descriptor: D fp32, A/B fp16 (0) or bf16 (1); M, N of the whole pair.
__device__ __forceinline__ uint32_t idesc2(int M, int N, uint32_t fmt, int b_mn_major) {
  return (1u << 4) | (fmt << 7) | (fmt << 10) | ((uint32_t)(b_mn_major & 1) << 16) | ((uint32_t)(N >> 3) << 17) |
         ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void mma2_ss(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void mma2_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on the barrier at the same offset in both CTAs of the pair when every
// MMA this thread issued before has completed.
__device__ __forceinline__ void commit2_both(uint32_t bar) {
  asm volatile(
      "{\n\t.reg .b16 m;\n\tmov.b16 m, 3;\n\t"
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], m;\n\t}" ::"r"(
          bar)
      : "memory");
}

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// The shared::cluster address of this CTA's shared location `addr` in CTA `rank`.
__device__ __forceinline__ uint32_t map_to_rank(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}

__device__ __forceinline__ void arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

__device__ __forceinline__ bool try_wait_cluster(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait with cluster-scope acquire (barriers other CTAs arrive on).
__device__ __forceinline__ bool wait_cluster_bounded(uint32_t bar, uint32_t parity) {
  if (try_wait_cluster(bar, parity)) return true;
  const long long t0 = clock64();
  while (true) {
    if (try_wait_cluster(bar, parity)) return true;
    if (clock64() - t0 > PA_WAIT_LIMIT_CYCLES) return false;
  }
}

// TMA tile load into this CTA's shared memory, the transaction bytes counted on
// the barrier at cluster address `bar` (CTA 0's barrier: the pair's MMA thread waits there).
__device__ __forceinline__ void tma_load_4d_pair(uint32_t dst, const CUtensorMap* map, uint32_t bar, int x, int y,
                                                 int z, int w) {
  asm volatile(
      "cp.async.bulk.tensor.4d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y), "r"(z), "r"(w)
      : "memory");
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_fence_before2() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tmem_fence_after2() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld32x(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_st32x(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]),
      "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]),
      "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

__device__ __forceinline__ void tmem_st8x(uint32_t taddr, const uint32_t* r) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr), "r"(r[0]),
               "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
               : "memory");
}

__device__ __forceinline__ void tmem_wait_ld2() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st2() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// p ~ hi + lo as bf16 pairs cut by truncation (see split_bf16_pair in pa_prefill_umma.cu).
__device__ __forceinline__ void split_pair2(float p0, float p1, uint32_t& hi, uint32_t& lo) {
  const uint32_t b0 = __float_as_uint(p0), b1 = __float_as_uint(p1);
  hi = __byte_perm(b0, b1, 0x7632);
  const float r0 = p0 - __uint_as_float(b0 & 0xffff0000u);
  const float r1 = p1 - __uint_as_float(b1 & 0xffff0000u);
  lo = __byte_perm(__float_as_uint(r0), __float_as_uint(r1), 0x7632);
}

__device__ __forceinline__ uint32_t sw128(int r, int c) { return (uint32_t)(r * 128 + ((c ^ (r & 7)) << 4)); }

}  // namespace

template <typename T>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(320, 1)
    prefill_umma2_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
                         const DecodeParams p) {
  constexpr bool kSplit = kSplitProbabilities<T>::value;
  constexpr uint32_t FMT = kFmt2<T>::value;
  constexpr int S = kStages2;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
  uint8_t* s_kv = smem;                   // [stage][K: 2 halves x 32 tokens | V: 64 tokens x this CTA's half]
  uint8_t* s_q = s_kv + S * STAGE_BYTES2;  // [tile][2 halves][128 rows x 128 B]
  uint64_t* bars = reinterpret_cast<uint64_t*>(s_q + 2 * QT_BYTES2);
  uint64_t* kv_full = bars;           // [S] (CTA 0's: both CTAs' loads of a chunk)
  uint64_t* kv_empty = kv_full + S;   // [S] (both CTAs': the pair's MMAs of the chunk done)
  uint64_t* s_full = kv_empty + S;    // [tile * 2 + buffer]
  uint64_t* p_full = s_full + 4;      // [tile * 2 + buffer] (CTA 0's: both CTAs' P written)
  uint64_t* pv_done = p_full + 4;     // [tile * 2 + buffer]
  uint64_t* q_ready = pv_done + 4;    // [1] (CTA 0's: both CTAs' Q in shared memory)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(q_ready + 1);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;

  // Pair -> (sequence, kv head, 512-row block); pairs of one (sequence, kv
  // head) adjacent, the latest rows first.
  const int cap = p.max_blocks * p.bs;
  const int MT = (p.GQ + 511) / 512;
  const int pair = (int)(blockIdx.x >> 1);
  const int mt = MT - 1 - pair % MT;
  const int bh = pair / MT;
  const int b = bh / p.Hkv;
  const int h = bh - b * p.Hkv;
  int L = p.context_lens[b] + p.len_offset;
  if (L > cap) {
    if (tid == 0 && leader && h == 0 && mt == MT - 1) raise_flag(p.status, PA_DEVERR_TABLE_UNDERRUN);
    L = cap;
  }
  if (L < 0) L = 0;
  const int prow0 = mt * 512;                       // first row of the pair
  const int prows = min(512, p.GQ - prow0);         // rows of the pair that exist
  const int lim_pair = L - p.q_len + (prow0 + prows - 1) / p.G;
  const int kv_end = L;
  const int n_chunks = lim_pair < 0 ? 0 : (lim_pair + kChunk2) / kChunk2;
  const int row0 = prow0 + (int)rank * 256;         // this CTA's first row

  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(smem_addr(&kv_full[s]), 1);
      mbar_init(smem_addr(&kv_empty[s]), 1);
    }
    for (int i = 0; i < 4; ++i) {
      mbar_init(smem_addr(&s_full[i]), 1);
      mbar_init(smem_addr(&p_full[i]), 8);  // four softmax warps in each CTA
      mbar_init(smem_addr(&pv_done[i]), 1);
    }
    mbar_init(smem_addr(q_ready), 16);  // the eight softmax warps of each CTA
    prefetch_tensormap(&tmk);
    prefetch_tensormap(&tmv);
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                 "r"(kTmemCols2)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  fence_mbar_init();
  tmem_fence_before2();
  cluster_sync_all();  // both CTAs' barriers and TMEM exist before anything crosses the pair
  tmem_fence_after2();
  const uint32_t tmem = *tmem_slot;
  pdl_wait_previous();

  // CTA 0's barriers, as cluster addresses (for CTA 1's loads and arrivals)
  const uint32_t kv_full0 = map_to_rank(smem_addr(&kv_full[0]), 0);
  const uint32_t p_full0 = map_to_rank(smem_addr(&p_full[0]), 0);
  const uint32_t q_ready0 = map_to_rank(smem_addr(q_ready), 0);

  if (warp == 8) {
    // ---------------- producer: this CTA's half of every K/V chunk ----------------
    int win_base = -1, win_val = -1;
    const int bs = p.bs;
    bool ok = true;
    for (int j = 0; j < n_chunks && ok; ++j) {
      const int stage = j % S;
      if (j >= S) {
        int w = 1;
        if (lane == 0) w = mbar_wait_bounded(smem_addr(&kv_empty[stage]), (uint32_t)(((j / S) - 1) & 1)) ? 1 : 0;
        w = __shfl_sync(0xffffffffu, w, 0);
        if (!w) {
          if (lane == 0) raise_flag(p.status, PA_DEVERR_WAIT_TIMEOUT);
          ok = false;
          break;
        }
      }
      const uint32_t base = smem_addr(s_kv + stage * STAGE_BYTES2);
      const uint32_t full = kv_full0 + (uint32_t)stage * 8u;
      const int chunk0 = j * kChunk2;
      const int units = min(4, (kv_end - chunk0 + 15) / 16);  // units of this chunk the sequence reaches
      {
        const int lb_first = chunk0 / bs, lb_last = (chunk0 + kChunk2 - 1) / bs;
        if (win_base < 0 || lb_first < win_base || lb_last >= win_base + 32) {
          win_base = lb_first;
          const int e = lb_first + lane;
          win_val = (e < p.max_blocks) ? __ldg(&p.block_tables[(long long)b * p.bt_stride + e]) : -1;
        }
      }
      // Boxes (2 KB each): lanes 0-3 K of this CTA's units (2 units x 2 halves),
      // lanes 4-7 V of this CTA's half for the chunk's 4 units.
      const bool is_v = lane >= 4 && lane < 8;
      const int u = is_v ? lane - 4 : (int)rank * 2 + (lane >> 1);
      const int hf = is_v ? (int)rank : (lane & 1);
      const int tok0 = chunk0 + u * 16;
      const int lb0 = tok0 / bs;
      const int ph = __shfl_sync(0xffffffffu, win_val, (lb0 - win_base) & 31);
      if (leader && lane == 0) mbar_arrive_expect_tx(smem_addr(&kv_full[stage]), (uint32_t)units * 8192u);
      __syncwarp();
      if (lane < 8 && u < units) {
        const uint32_t dst = is_v ? base + K_BYTES + (uint32_t)u * 2048u
                                  : base + (uint32_t)hf * K_HALF_BYTES + (uint32_t)(u - (int)rank * 2) * 2048u;
        if (!is_v && hf == 0 && (ph < 0 || ph >= p.num_blocks)) raise_flag(p.status, PA_DEVERR_BLOCK_ID_RANGE);
        tma_load_4d_pair(dst, is_v ? &tmv : &tmk, full, hf * 64, tok0 - lb0 * bs, h, ph);
      }
      __syncwarp();
    }
  } else if (warp == 9) {
    // ---------------- MMA issue (one thread of CTA 0 for the pair) ----------------
    if (leader && lane == 0 && n_chunks > 0) {
      bool ok = wait_cluster_bounded(smem_addr(q_ready), 0);
      const uint32_t id_s = idesc2(256, kChunk2, FMT, 0);
      const uint32_t id_o = idesc2(256, D2, FMT, 1);
      const uint64_t qdesc[2] = {desc_sw128(smem_addr(s_q), 16, 1024), desc_sw128(smem_addr(s_q + QT_BYTES2), 16, 1024)};
      const uint64_t kdesc0 = desc_sw128(smem_addr(s_kv), 16, 1024);
      const uint64_t vdesc0 = desc_sw128(smem_addr(s_kv) + K_BYTES, 16, 1024);
      auto qk = [&](int t, int jq) {  // S_t(jq) = Q_t K(jq)^T for the pair
        const uint64_t kd = kdesc0 + (uint64_t)(((jq % S) * STAGE_BYTES2) >> 4);
        const uint32_t d = tmem + (uint32_t)(t * 256 + (jq & 1) * kChunk2);
#pragma unroll
        for (int ks = 0; ks < D2 / 16; ++ks) {
          const uint64_t sq = (uint64_t)(((ks >> 2) * 16384u + (ks & 3) * 32u) >> 4);
          const uint64_t sk = (uint64_t)(((ks >> 2) * K_HALF_BYTES + (ks & 3) * 32u) >> 4);
          mma2_ss(d, qdesc[t] + sq, kd + sk, id_s, ks > 0 ? 1u : 0u);
        }
      };
      auto pv = [&](int t, int jp) {  // O_t += P_t(jp) V(jp) for the pair
        const uint64_t vb = vdesc0 + (uint64_t)(((jp % S) * STAGE_BYTES2) >> 4);
        const uint32_t pcol = tmem + (uint32_t)(t * 256 + (jp & 1) * kChunk2);
        const uint32_t o = tmem + (uint32_t)(t * 256 + 128);
#pragma unroll
        for (int ks = 0; ks < kChunk2 / 16; ++ks) {
          const uint64_t vd = vb + (uint64_t)((ks * 2048u) >> 4);
          mma2_ts(o, pcol + ks * 8u, vd, id_o, (jp > 0 || ks > 0) ? 1u : 0u);
          if (kSplit) mma2_ts(o, pcol + 32u + ks * 8u, vd, id_o, 1u);
        }
      };
      int pend_t = -1, pend_j = 0;
      auto flush = [&]() {
        if (pend_t >= 0) {
          commit2_both(smem_addr(&pv_done[pend_t * 2 + (pend_j & 1)]));
          commit2_both(smem_addr(&kv_empty[pend_j % S]));
          pend_t = -1;
        }
      };
      if (ok) ok = wait_cluster_bounded(smem_addr(&kv_full[0]), 0);
      if (ok) {
        tmem_fence_after2();
        qk(0, 0);
        qk(1, 0);
        commit2_both(smem_addr(&s_full[0]));
        commit2_both(smem_addr(&s_full[2]));
      }
      for (int j = 0; j < n_chunks && ok; ++j) {
        const int jn = j + 1;
        if (jn < n_chunks) {
          ok = wait_cluster_bounded(smem_addr(&kv_full[jn % S]), (uint32_t)((jn / S) & 1));
          flush();
          if (!ok) break;
          qk(0, jn);
          qk(1, jn);
        } else {
          flush();
        }
        ok = wait_cluster_bounded(smem_addr(&p_full[j & 1]), (uint32_t)((j >> 1) & 1));
        if (jn < n_chunks) {
          commit2_both(smem_addr(&s_full[jn & 1]));
          commit2_both(smem_addr(&s_full[2 + (jn & 1)]));
        }
        if (!ok) break;
        tmem_fence_after2();
        pv(0, j);
        ok = wait_cluster_bounded(smem_addr(&p_full[2 + (j & 1)]), (uint32_t)((j >> 1) & 1));
        commit2_both(smem_addr(&pv_done[j & 1]));
        if (!ok) break;
        tmem_fence_after2();
        pv(1, j);
        pend_t = 1;
        pend_j = j;
      }
      flush();
      if (!ok) raise_flag(p.status, PA_DEVERR_WAIT_TIMEOUT);
    }
    __syncwarp();
  } else {
    // ---------------- softmax warps: tile t, thread = query row = TMEM lane ----------------
    const int t = warp >> 2;
    const int r = (warp & 3) * 32 + lane;
    const int qr = row0 + t * 128 + r;
    const bool row_ok = qr < p.GQ;
    const int tq = row_ok ? qr / p.G : 0;
    const int g = row_ok ? qr - tq * p.G : 0;
    const int lim = row_ok ? L - p.q_len + tq : -1;  // last attendable position of this row
    {
      const T* qrow = static_cast<const T*>(p.q) + (long long)b * p.q_sb + (long long)(h * p.G + g) * p.q_sh +
                      (long long)tq * p.q_st;
      uint8_t* qt = s_q + t * QT_BYTES2;
#pragma unroll
      for (int c = 0; c < D2 / 8; ++c) {
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (row_ok && c * 8 < p.Dv) v = *reinterpret_cast<const uint4*>(qrow + c * 8);
        *reinterpret_cast<uint4*>(qt + (c >> 3) * 16384 + sw128(r, c & 7)) = v;
      }
    }
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) arrive_cluster(q_ready0);

    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    const uint32_t t_s = tmem + (uint32_t)(t * 256) + lane_base;
    const uint32_t t_o = t_s + 128u;
    float m_ref = -INFINITY;
    float l = 0.f;
    bool ok = true;
    for (int j = 0; j < n_chunks; ++j) {
      const int sb = j & 1;
      if (!mbar_test_then_wait(smem_addr(&s_full[t * 2 + sb]), (uint32_t)((j >> 1) & 1))) {
        ok = false;
        break;
      }
      tmem_fence_after2();
      float x[kChunk2];
      {
        uint32_t r0[32], r1[32];
        tmem_ld32x(t_s + sb * kChunk2, r0);
        tmem_ld32x(t_s + sb * kChunk2 + 32, r1);
        tmem_wait_ld2();
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          x[i] = __uint_as_float(r0[i]);
          x[32 + i] = __uint_as_float(r1[i]);
        }
      }
      const int tok0 = j * kChunk2;
      if (tok0 + kChunk2 - 1 > lim) {
#pragma unroll
        for (int i = 0; i < kChunk2; ++i)
          if (tok0 + i > lim) x[i] = -INFINITY;
      }
      float mx_raw = -INFINITY;
#pragma unroll
      for (int i = 0; i < kChunk2; ++i) mx_raw = fmaxf(mx_raw, x[i]);
      const float sl2 = p.scale_log2;
      const float mx = mx_raw * sl2;
      float alpha = 1.f;
      bool move = false;
      if (mx > m_ref + kRescaleThreshold2 || (m_ref == -INFINITY && mx != -INFINITY)) {
        alpha = (m_ref == -INFINITY) ? 0.f : ex2(m_ref - mx);
        m_ref = mx;
        move = true;
      }
      const float nbase = (m_ref == -INFINITY) ? 0.f : -m_ref;
      if (__any_sync(0xffffffffu, move && j > 0)) {
        if (!mbar_wait_bounded(smem_addr(&pv_done[t * 2 + ((j - 1) & 1)]), (uint32_t)(((j - 1) >> 1) & 1))) {
          ok = false;
          break;
        }
        tmem_fence_after2();
        const float a = (move && j > 0) ? alpha : 1.f;
#pragma unroll
        for (int c0 = 0; c0 < D2; c0 += 32) {
          uint32_t o[32];
          tmem_ld32x(t_o + c0, o);
          tmem_wait_ld2();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * a);
          tmem_st32x(t_o + c0, o);
        }
      }
      float ps = 0.f;
#pragma unroll
      for (int piece = 0; piece < 4; ++piece) {
        uint32_t hi[8], lo[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float p0 = ex2(fmaf(x[16 * piece + 2 * i], sl2, nbase));
          const float p1 = ex2(fmaf(x[16 * piece + 2 * i + 1], sl2, nbase));
          ps += p0 + p1;
          if constexpr (kSplit) {
            split_pair2(p0, p1, hi[i], lo[i]);
          } else {
            hi[i] = pack2<T>(p0, p1);
            lo[i] = 0u;
          }
        }
        tmem_st8x(t_s + sb * kChunk2 + piece * 8, hi);
        if (kSplit) tmem_st8x(t_s + sb * kChunk2 + 32 + piece * 8, lo);
      }
      l = l * alpha + ps;
      // Tail chunk: this CTA's V half holds stale rows at or past kv_end (P is
      // 0 there, but 0 * NaN is not); tile 0's warps zero them before their P
      // is published, and tile 1's P.V is issued after tile 0's.
      const int valid = kv_end - tok0;
      if (t == 0 && valid < kChunk2) {
        uint8_t* vbase = s_kv + (j % S) * STAGE_BYTES2 + K_BYTES;
        const int nrows = kChunk2 - valid;
        for (int i = r; i < nrows * 8; i += 128) {
          const int row = valid + i / 8;
          *reinterpret_cast<uint4*>(vbase + row * 128 + (i & 7) * 16) = make_uint4(0u, 0u, 0u, 0u);
        }
        fence_proxy_async_smem();
      }
      tmem_wait_st2();
      tmem_fence_before2();
      __syncwarp();
      if (lane == 0) arrive_cluster(p_full0 + (uint32_t)(t * 2 + sb) * 8u);
    }

    // ---- epilogue ----
    if (ok && n_chunks > 0) {
      const int jl = n_chunks - 1;
      ok = mbar_wait_bounded(smem_addr(&pv_done[t * 2 + (jl & 1)]), (uint32_t)((jl >> 1) & 1));
    }
    if (!ok && lane == 0) raise_flag(p.status, PA_DEVERR_WAIT_TIMEOUT);
    tmem_fence_after2();
    T* orow = static_cast<T*>(p.out) + (long long)b * p.o_sb + (long long)(h * p.G + g) * p.o_sh +
              (long long)tq * p.o_st;
    const float inv = (ok && l > 0.f) ? 1.f / l : 0.f;
#pragma unroll
    for (int c0 = 0; c0 < D2; c0 += 32) {
      uint32_t o[32];
      if (n_chunks > 0) {
        tmem_ld32x(t_o + c0, o);
        tmem_wait_ld2();
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) o[i] = 0u;
      }
      if (row_ok) {
#pragma unroll
        for (int i = 0; i < 32; i += 8) {
          if (c0 + i >= p.Dv) break;
          uint4 v;
          v.x = pack2<T>(__uint_as_float(o[i]) * inv, __uint_as_float(o[i + 1]) * inv);
          v.y = pack2<T>(__uint_as_float(o[i + 2]) * inv, __uint_as_float(o[i + 3]) * inv);
          v.z = pack2<T>(__uint_as_float(o[i + 4]) * inv, __uint_as_float(o[i + 5]) * inv);
          v.w = pack2<T>(__uint_as_float(o[i + 6]) * inv, __uint_as_float(o[i + 7]) * inv);
          *reinterpret_cast<uint4*>(orow + c0 + i) = v;
        }
      }
    }
  }

  // Neither CTA releases TMEM (or leaves, taking its shared memory with it)
  // while the pair's MMAs or the other CTA's reads may still run.
  tmem_fence_before2();
  cluster_sync_all();
  if (warp == 0) {
    tmem_fence_after2();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols2) : "memory");
  }
}

size_t prefill_umma2_smem_bytes() { return 1024 + (size_t)kStages2 * STAGE_BYTES2 + 2 * QT_BYTES2 + 256; }

template <typename T>
static cudaError_t launch_umma2_impl(const DecodeParams& p, const CUtensorMap& tmk, const CUtensorMap& tmv, bool pdl,
                                     cudaStream_t stream) {
  const size_t smem = prefill_umma2_smem_bytes();
  static bool prepared[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !prepared[dev]) {
    cudaError_t e =
        cudaFuncSetAttribute(prefill_umma2_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    prepared[dev] = true;
  }
  const long long pairs = (long long)p.B * p.Hkv * ((p.GQ + 511) / 512);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(2 * pairs));
  cfg.blockDim = dim3(320);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = pdl ? attr : nullptr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, prefill_umma2_kernel<T>, tmk, tmv, p);
}

cudaError_t launch_prefill_umma2(const DecodeParams& p, const CUtensorMap& tmk, const CUtensorMap& tmv, int dtype,
                                 bool pdl, cudaStream_t stream) {
  if (p.D != D2 || p.bs < 16) return cudaErrorInvalidValue;
  if (dtype == PA_DTYPE_BFLOAT16) return launch_umma2_impl<__nv_bfloat16>(p, tmk, tmv, pdl, stream);
  if (dtype == PA_DTYPE_FLOAT16) return launch_umma2_impl<__half>(p, tmk, tmv, pdl, stream);
  return cudaErrorInvalidValue;
}

}  // namespace pa
