// pa_prefill_umma.cu — multi-query attention over paged KV on 5th-generation
// tensor cores (tcgen05 / UMMA, accumulators in TMEM), fp16 / bf16, sm_100a.
//
// Same contract and row layout as the other decode kernels: rows of one KV head
// are token-major (row r = query token r / G of head h*G + r % G); query token t
// attends positions 0 .. L - q_len + t.  A CTA owns 256 rows -- two 128-row
// MMA tiles -- of one (sequence, kv head) and streams the sequence's K/V in
// 64-token chunks shared by both tiles.  The CTAs of one (sequence, kv head)
// are adjacent in the grid, so they run in one wave and share K/V through L2.
//
//   warp 8 (producer)   TMA-loads each chunk's four 16-token units (K and V, two
//                       64-column halves each, 128-byte swizzle) into a ring,
//                       every box of a chunk from its own lane in one
//                       instruction;
//   warp 9 (MMA)        one thread issues, per chunk, S_t = Q_t K^T (M=128, N=64,
//                       K=D) for both tiles into TMEM, then O_t += P_t V
//                       (M=128, N=D, K=64) with P_t read from TMEM, signalling
//                       mbarriers with tcgen05.commit (each commit after its
//                       next barrier check: a check right behind a commit
//                       stalls while the queued MMAs drain);
//   warps 0-3 / 4-7     softmax of tile 0 / tile 1: thread i owns query row i
//                       = TMEM lane i; it loads its S row (tcgen05.ld), masks,
//                       takes the max and exponentials without any cross-thread
//                       reduction, and writes its P row (bf16: hi and lo parts,
//                       so P.V keeps ~16 bits of P) back over the same TMEM
//                       columns (tcgen05.st) as the A operand of the PV MMA;
//                       finally it reads O back, normalises and stores it;
//   warp 10             (the cascade's prefix pass only) checks that every
//                       member reaches the shared prefix through the same
//                       physical blocks.
//
// While one tile's softmax runs, the tensor core works on the other tile's
// products, so neither waits for the other.  Each tile has two S/P buffers in
// TMEM; the MMA thread refills a buffer right after issuing the PV that reads
// its P (the tensor core runs one thread's MMAs in issue order).  The online
// softmax keeps a reference max per row and rescales O (TMEM load, scale,
// store) only when a chunk raises the row max by more than 2^8, so p stays
// below 256 and the arithmetic is exact; most chunks skip the rescale.  Every
// wait is bounded; TMEM is always released before the CTA exits.
#include <math.h>

#include "pa_common.cuh"
#include "pa_internal.h"
#include "pa_tile_math.cuh"

namespace pa {

namespace {

constexpr int kChunk = kUmmaChunkTokens;  // tokens per chunk (N of the QK^T MMA)
constexpr uint32_t kTmemCols = 512;        // per tile: S/P buffers (2 x 64) + O (<= 128), at column 256 * tile
constexpr int kTileRows = kUmmaTileRows;   // query rows per CTA (two 128-row MMA tiles)
constexpr float kRescaleThreshold = 8.f;   // log2 units: rescale when the max grows by > 2^8

// K/V chunks in flight: as many as the shared memory left after Q allows.
template <int D>
struct kUmmaStages {
  static constexpr int value = D == 128 ? 4 : 8;
};

// UMMA A/B element format code of kind::f16: 0 = fp16, 1 = bf16.
template <typename T>
struct kUmmaFormat;
template <>
struct kUmmaFormat<__half> {
  static constexpr uint32_t value = 0;
};
template <>
struct kUmmaFormat<__nv_bfloat16> {
  static constexpr uint32_t value = 1;
};

__device__ __forceinline__ uint64_t umma_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((addr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;  // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;  // 128-byte swizzle
  return d;
}

// kind::f16 instruction descriptor: D fp32, A/B fp16 (fmt 0) or bf16 (fmt 1).
__device__ __forceinline__ uint32_t umma_idesc(int M, int N, uint32_t ab_fmt, int b_mn_major) {
  return (1u << 4) | (ab_fmt << 7) | (ab_fmt << 10) | ((uint32_t)(b_mn_major & 1) << 16) |
         ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Same with the A operand (M x K, K-major: row m in TMEM lane m, two 16-bit
// elements per 32-bit column) read from tensor memory.
__device__ __forceinline__ void umma_f16_tmem_a(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                                uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}

__device__ __forceinline__ void tmem_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tmem_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]),
      "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]),
      "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t* r) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr), "r"(r[0]),
               "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
               : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Two probabilities (>= 0) as packed bf16 pairs hi and lo with p ~ hi + lo,
// both by truncation with bit operations: hi keeps the upper 16 bits of p, lo
// those of the exact fp32 residual p - hi.  hi + lo carries about 15 bits of p
// (relative error below 2^-15) and, unlike round-to-nearest conversions, takes
// no conversion instructions, which share the exp2 unit's throughput.
__device__ __forceinline__ void split_bf16_pair(float p0, float p1, uint32_t& hi, uint32_t& lo) {
  const uint32_t b0 = __float_as_uint(p0), b1 = __float_as_uint(p1);
  hi = __byte_perm(b0, b1, 0x7632);  // low half: p0's upper 16 bits; high half: p1's
  const float r0 = p0 - __uint_as_float(b0 & 0xffff0000u);
  const float r1 = p1 - __uint_as_float(b1 & 0xffff0000u);
  lo = __byte_perm(__float_as_uint(r0), __float_as_uint(r1), 0x7632);
}

// Byte offset of 16-byte chunk `c` of row `r` in a 128-byte-swizzled region.
__device__ __forceinline__ uint32_t sw128_chunk(int r, int c) { return (uint32_t)(r * 128 + ((c ^ (r & 7)) << 4)); }

}  // namespace

// kPrefix = false: a CTA owns 256 rows of one (sequence, kv head) and writes
// normalised output rows.  kPrefix = true (the prefix part of
// pa_decode_cascade): a CTA owns 256 of the member rows of one (split, prefix
// group, kv head) -- row r is row r % GQ of member r / GQ -- attends the
// group's shared blocks in the split's token range through the first member's
// block table, and leaves (m, l, unnormalised O) per row.
template <typename T, int D, bool kPrefix>
__global__ void __launch_bounds__(umma_threads(kPrefix), 1)
    prefill_umma_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
                        const DecodeParams p) {
  constexpr int HALVES = D / 64;
  constexpr int S = kUmmaStages<D>::value;
  constexpr uint32_t HALF_BYTES = kChunk * 128;          // 64 rows x 128 B
  constexpr uint32_t KV_BYTES = 2 * HALVES * HALF_BYTES;  // K and V of one chunk
  constexpr uint32_t QT_BYTES = HALVES * 128 * 128;       // one 128-row tile of Q
  constexpr bool kSplit = kSplitProbabilities<T>::value;
  constexpr uint32_t FMT = kUmmaFormat<T>::value;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
  uint8_t* s_kv = smem;                  // [stage][K halves | V halves]
  uint8_t* s_q = s_kv + S * KV_BYTES;    // [tile][halves][128 rows x 128 B]
  uint64_t* bars = reinterpret_cast<uint64_t*>(s_q + 2 * QT_BYTES);
  uint64_t* kv_full = bars;              // [S]
  uint64_t* kv_empty = kv_full + S;      // [S]
  uint64_t* s_full = kv_empty + S;       // [tile * 2 + buffer]: S of a chunk is in TMEM
  uint64_t* p_full = s_full + 4;         // [tile * 2 + buffer]: P of a chunk is in TMEM
  uint64_t* pv_done = p_full + 4;        // [tile * 2 + buffer]: the PV reading that P completed
  uint64_t* q_ready = pv_done + 4;       // [1]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(q_ready + 1);
  __shared__ int s_last;

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;

  const int cap = p.max_blocks * p.bs;
  // CTA: the sequence whose block table is read (b_kv), the kv head, the first
  // row, the rows that exist, and the token range [kv_lo, kv_end) streamed in
  // n_chunks chunks (tokens at or past kv_end are never attended).
  int b_kv, h, row0, rows_total, kv_lo, kv_end, n_chunks;
  int moff = 0, split = 0, prefix_tokens = 0, tile_id = 0;
  if constexpr (kPrefix) {
    const int MT = (p.max_members * p.GQ + kTileRows - 1) / kTileRows;
    int idx = (int)blockIdx.x;
    const int mt = idx % MT;
    idx /= MT;
    h = idx % p.Hkv;
    idx /= p.Hkv;
    const int gi = idx % p.num_groups;
    split = idx / p.num_groups;
    tile_id = (gi * p.Hkv + h) * MT + mt;
    moff = p.member_off[gi];
    int nmem = p.member_off[gi + 1] - moff;
    if (nmem > p.max_members || p.group_prefix[gi] > p.max_prefix) {
      if (tid == 0 && h == 0 && mt == 0 && split == 0) raise_flag(p.status, PA_DEVERR_PREFIX);
      nmem = min(nmem, p.max_members);
    }
    if (nmem < 0) nmem = 0;
    prefix_tokens = cascade_prefix_tokens(p, gi);
    rows_total = nmem * p.GQ;
    row0 = mt * kTileRows;
    kv_lo = split * p.split_tokens;
    kv_end = min(prefix_tokens, kv_lo + p.split_tokens);
    b_kv = nmem > 0 ? p.member_seq[moff] : 0;
    if (b_kv < 0 || b_kv >= p.B) {  // the group's table row must be a batch row
      if (tid == 0) raise_flag(p.status, PA_DEVERR_PREFIX);
      b_kv = 0;
      rows_total = 0;
    }
    n_chunks = (row0 < rows_total && kv_end > kv_lo) ? (kv_end - kv_lo + kChunk - 1) / kChunk : 0;
  } else {
    const int MT = (p.GQ + kTileRows - 1) / kTileRows;
    // The CTAs of one (sequence, kv head) read the same K/V: adjacent block
    // indices put them in the same wave, so all but the first read hit L2.
    // Within a (sequence, kv head), the latest (heaviest) row blocks first.
    const int mt = MT - 1 - (int)(blockIdx.x % MT);
    const int bh = (int)(blockIdx.x / MT);
    b_kv = bh / p.Hkv;
    h = bh - b_kv * p.Hkv;
    int L = p.context_lens[b_kv] + p.len_offset;
    if (L > cap) {
      if (tid == 0 && h == 0 && mt == MT - 1) raise_flag(p.status, PA_DEVERR_TABLE_UNDERRUN);
      L = cap;
    }
    if (L < 0) L = 0;
    row0 = mt * kTileRows;
    rows_total = p.GQ;
    const int rows_cta = min(kTileRows, p.GQ - row0);
    const int lim_cta = L - p.q_len + (row0 + rows_cta - 1) / p.G;
    kv_lo = 0;
    kv_end = L;
    n_chunks = lim_cta < 0 ? 0 : (lim_cta + kChunk) / kChunk;
  }
  const int ntiles = (row0 + 128 < rows_total) ? 2 : 1;  // MMA tiles holding rows

  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(smem_addr(&kv_full[s]), 1);
      mbar_init(smem_addr(&kv_empty[s]), 1);
    }
    for (int i = 0; i < 4; ++i) {
      mbar_init(smem_addr(&s_full[i]), 1);
      mbar_init(smem_addr(&p_full[i]), 4);
      mbar_init(smem_addr(&pv_done[i]), 1);
    }
    mbar_init(smem_addr(q_ready), 8);
    prefetch_tensormap(&tmk);
    prefetch_tensormap(&tmv);
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  fence_mbar_init();
  tmem_fence_before();
  __syncthreads();
  tmem_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_wait_previous();
  // The cascade's decode kernel may start its prologue now; it waits for this
  // grid to finish before reading the prefix states.
  if constexpr (kPrefix) pdl_launch_dependents();

  if (warp == 8) {
    // ---------------- producer: K/V chunks by TMA ----------------
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
      const uint32_t base = smem_addr(s_kv + stage * KV_BYTES);
      const uint32_t bar = smem_addr(&kv_full[stage]);
      const int chunk0 = kv_lo + j * kChunk;
      // units of this chunk the token range reaches
      const int units = min(4, (kv_end - chunk0 + 15) / 16);
      // block-table window (32 entries, one per lane) covering every block of the chunk
      {
        const int lb_first = chunk0 / bs, lb_last = (chunk0 + kChunk - 1) / bs;
        if (win_base < 0 || lb_first < win_base || lb_last >= win_base + 32) {
          win_base = lb_first;
          const int e = lb_first + lane;
          win_val = (e < p.max_blocks) ? __ldg(&p.block_tables[(long long)b_kv * p.bt_stride + e]) : -1;
        }
      }
      // Lane -> (unit, K or V, 64-column half): every box of the chunk is issued
      // by its own lane in one instruction.  A single thread issuing them one
      // after another keeps only about one chunk in flight.
      const int u = lane / (2 * HALVES);
      const int is_v = (lane / HALVES) & 1;
      const int hf = lane % HALVES;
      const int tok0 = chunk0 + u * 16;
      const int lb0 = tok0 / bs;
      const int ph0 = __shfl_sync(0xffffffffu, win_val, (lb0 - win_base) & 31);
      const int ph1 = __shfl_sync(0xffffffffu, win_val, (lb0 + 1 - win_base) & 31);
      if (lane == 0) {
        uint32_t tx = 0;
        for (int v = 0; v < units; ++v) {
          const int t0 = chunk0 + v * 16;
          if (bs >= 16) {
            tx += 2u * HALVES * 2048u;
          } else {
            const bool need1 = (t0 / bs + 1) * bs < kv_end;
            tx += (need1 ? 2u : 1u) * 2u * HALVES * (uint32_t)bs * 128u;
          }
        }
        mbar_arrive_expect_tx(bar, tx);
      }
      __syncwarp();
      if (u < units) {
        const CUtensorMap* map = is_v ? &tmv : &tmk;
        const uint32_t dst = base + (uint32_t)(is_v * HALVES + hf) * HALF_BYTES + (uint32_t)u * 2048u;
        const bool check = !is_v && hf == 0;
        if (bs >= 16) {
          if (check && (ph0 < 0 || ph0 >= p.num_blocks)) raise_flag(p.status, PA_DEVERR_BLOCK_ID_RANGE);
          tma_load_4d(dst, map, bar, hf * 64, tok0 - lb0 * bs, h, ph0);
        } else {
          const bool need1 = (lb0 + 1) * bs < kv_end;
          if (check && (ph0 < 0 || ph0 >= p.num_blocks || (need1 && (ph1 < 0 || ph1 >= p.num_blocks))))
            raise_flag(p.status, PA_DEVERR_BLOCK_ID_RANGE);
          tma_load_4d(dst, map, bar, hf * 64, 0, h, ph0);
          if (need1) tma_load_4d(dst + (uint32_t)bs * 128u, map, bar, hf * 64, 0, h, ph1);
        }
      }
      __syncwarp();
    }
  } else if (warp == 9) {
    // ---------------- MMA issue (one thread) ----------------
    if (lane == 0 && n_chunks > 0) {
      bool ok = mbar_wait_bounded(smem_addr(q_ready), 0);
      const uint32_t id_s = umma_idesc(128, kChunk, FMT, 0);
      const uint32_t id_o = umma_idesc(128, D, FMT, 1);
      // Descriptors built once per buffer; a k-step only advances the start
      // address field (addresses stay below 256 KB: no carry out of it).
      const uint64_t qdesc[2] = {umma_desc(smem_addr(s_q), 16, 1024), umma_desc(smem_addr(s_q + QT_BYTES), 16, 1024)};
      const uint64_t kdesc0 = umma_desc(smem_addr(s_kv), 16, 1024);
      const uint64_t vdesc0 = umma_desc(smem_addr(s_kv) + HALVES * HALF_BYTES, HALF_BYTES, 1024);
      auto qk_mmas = [&](int t, int jq) {  // S_t(jq) = Q_t K(jq)^T
        const uint64_t kd = kdesc0 + (uint64_t)(((jq % S) * KV_BYTES) >> 4);
        const uint32_t d = tmem + (uint32_t)(t * 256 + (jq & 1) * kChunk);
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks) {
          const uint64_t step_q = (uint64_t)(((ks >> 2) * 16384u + (ks & 3) * 32u) >> 4);
          const uint64_t step_k = (uint64_t)(((ks >> 2) * HALF_BYTES + (ks & 3) * 32u) >> 4);
          umma_f16(d, qdesc[t] + step_q, kd + step_k, id_s, ks > 0 ? 1u : 0u);
        }
      };
      auto pv_mmas = [&](int t, int jp) {  // O_t += P_t(jp) V(jp)
        const uint64_t vb = vdesc0 + (uint64_t)(((jp % S) * KV_BYTES) >> 4);
        const uint32_t pcol = tmem + (uint32_t)(t * 256 + (jp & 1) * kChunk);  // P hi: +0..31, lo: +32..63
        const uint32_t o = tmem + (uint32_t)(t * 256 + 128);
#pragma unroll
        for (int ks = 0; ks < kChunk / 16; ++ks) {
          const uint64_t vd = vb + (uint64_t)((ks * 2048u) >> 4);
          umma_f16_tmem_a(o, pcol + ks * 8u, vd, id_o, (jp > 0 || ks > 0) ? 1u : 0u);
          if (kSplit) umma_f16_tmem_a(o, pcol + 32u + ks * 8u, vd, id_o, 1u);
        }
      };
      // Each group's commit is issued after this thread's next barrier check,
      // not before it: a check right behind a commit costs ~300 cycles of
      // this thread while the queued MMAs drain, one behind plain MMA issues
      // much less.  A commit tracks every MMA issued before it either way.
      int pend_t = -1, pend_j = 0;  // P.V of tile pend_t, chunk pend_j: its commits still to issue
      auto flush = [&]() {
        if (pend_t >= 0) {
          umma_commit(smem_addr(&pv_done[pend_t * 2 + (pend_j & 1)]));
          umma_commit(smem_addr(&kv_empty[pend_j % S]));  // both tiles' P.V of the stage issued
          pend_t = -1;
        }
      };
      // S of chunk j+1 (both tiles) is issued before P.V of chunk j, so a
      // tile's softmax of j+1 overlaps the products of chunk j.
      if (ok) ok = mbar_wait_bounded(smem_addr(&kv_full[0]), 0);
      if (ok) {
        tmem_fence_after();
        qk_mmas(0, 0);
        if (ntiles > 1) qk_mmas(1, 0);
        umma_commit(smem_addr(&s_full[0]));
        if (ntiles > 1) umma_commit(smem_addr(&s_full[2]));
      }
      for (int j = 0; j < n_chunks && ok; ++j) {
        const int jn = j + 1;
        if (jn < n_chunks) {
          ok = mbar_test_then_wait(smem_addr(&kv_full[jn % S]), (uint32_t)((jn / S) & 1));
          flush();
          if (!ok) break;
          // The buffer's previous P (chunk jn - 2) is read by a P.V this
          // thread issued before; tcgen05.mma operations of one thread run in
          // issue order, so S of chunk jn can go into it at once.  No tcgen05
          // fence here (one costs ~100 cycles of this thread's issue): the
          // softmax's reads of that buffer were ordered before this thread's
          // MMAs by the fence after the P wait of that P.V, and K is ordered
          // by its full barrier like any TMA-fed operand.  The tile index is a
          // literal in each call, so the descriptors are fixed at compile time.
          qk_mmas(0, jn);
          if (ntiles > 1) qk_mmas(1, jn);
        } else {
          flush();
        }
        ok = mbar_test_then_wait(smem_addr(&p_full[j & 1]), (uint32_t)((j >> 1) & 1));
        if (jn < n_chunks) {
          umma_commit(smem_addr(&s_full[jn & 1]));
          if (ntiles > 1) umma_commit(smem_addr(&s_full[2 + (jn & 1)]));
        }
        if (!ok) break;
        tmem_fence_after();
        pv_mmas(0, j);
        if (ntiles > 1) {
          ok = mbar_test_then_wait(smem_addr(&p_full[2 + (j & 1)]), (uint32_t)((j >> 1) & 1));
          umma_commit(smem_addr(&pv_done[j & 1]));
          if (!ok) break;
          tmem_fence_after();
          pv_mmas(1, j);
          pend_t = 1;
        } else {
          pend_t = 0;
        }
        pend_j = j;
      }
      flush();
      if (!ok) raise_flag(p.status, PA_DEVERR_WAIT_TIMEOUT);
    }
    __syncwarp();
  } else if (warp == 10) {
    // ---------------- prefix pass: member table check ----------------
    // Every member must reach the shared prefix through the same physical
    // blocks as the first member, whose table the producer reads.  The
    // split-0 / head-0 CTA holding a member's first row checks it, in this
    // warp of its own so the loads overlap the pipeline.  Member ids come 32 at
    // a time and every table load of a pass is independent.
    if constexpr (kPrefix) {
      if (split == 0 && h == 0 && prefix_tokens > 0 && row0 < rows_total) {
        const int i_lo = (row0 + p.GQ - 1) / p.GQ;
        const int i_end = (min(rows_total, row0 + kTileRows) + p.GQ - 1) / p.GQ;  // members i_lo .. i_end - 1
        const int nblk = (prefix_tokens + p.bs - 1) / p.bs;
        const int* first = p.block_tables + (long long)b_kv * p.bt_stride;
        bool bad = false;
        for (int m0 = i_lo; m0 < i_end; m0 += 32) {
          const int my_member = m0 + lane < i_end ? p.member_seq[moff + m0 + lane] : b_kv;
          const int nm = min(32, i_end - m0);
          for (int k0 = 0; k0 < nblk; k0 += 32) {
            const int k = k0 + lane;
            const bool kin = k < nblk;
            const int f = kin ? __ldg(first + k) : 0;
#pragma unroll 8
            for (int jm = 0; jm < nm; ++jm) {
              const int bm = __shfl_sync(0xffffffffu, my_member, jm);
              const bool valid = bm >= 0 && bm < p.B;
              const int e = (kin && valid && bm != b_kv) ? __ldg(p.block_tables + (long long)bm * p.bt_stride + k) : f;
              bad |= !valid || e != f;
            }
          }
        }
        if (__any_sync(0xffffffffu, bad) && lane == 0) raise_flag(p.status, PA_DEVERR_PREFIX);
      }
    }
  } else {
    // ---------------- softmax warps: tile t, thread = query row = TMEM lane ----------------
    const int t = warp >> 2;             // MMA tile of this warpgroup
    const int r = (warp & 3) * 32 + lane;  // row within the tile = TMEM lane
    const bool tile_on = t < ntiles;
    const int qr = row0 + t * 128 + r;
    const bool row_ok = tile_on && qr < rows_total;
    int tq = 0, g = 0, b = b_kv;
    int lim = -1;  // last attendable position of this row
    if (row_ok) {
      int r_in = qr;
      if constexpr (kPrefix) {
        const int i = qr / p.GQ;
        r_in = qr - i * p.GQ;
        b = p.member_seq[moff + i];
        if (b < 0 || b >= p.B) b = b_kv;  // flagged by the table check
      }
      tq = r_in / p.G;
      g = r_in - tq * p.G;
      const int Lb = min(max(p.context_lens[b] + p.len_offset, 0), cap);
      lim = Lb - p.q_len + tq;
      if constexpr (kPrefix) lim = min(lim, kv_end - 1);
    }
    // Q rows -> swizzled K-major tile t.  The warp loads its 32 rows together,
    // whole rows per instruction (a row's 16-byte pieces from consecutive
    // lanes), so each load touches a few full lines instead of one line per lane.
    {
      const T* qrow = static_cast<const T*>(p.q) + (long long)b * p.q_sb + (long long)(h * p.G + g) * p.q_sh +
                      (long long)tq * p.q_st;
      uint8_t* qt = s_q + t * QT_BYTES;
      constexpr int CH = D / 8;     // 16-byte pieces per row
      constexpr int RPI = 32 / CH;  // rows per warp instruction
      const int sub = lane / CH, c = lane % CH;
      const unsigned long long my_row = reinterpret_cast<unsigned long long>(qrow);
      uint4 v[32 / RPI];
#pragma unroll
      for (int k = 0; k < 32 / RPI; ++k) {
        const int src = k * RPI + sub;  // the lane whose row this is
        const T* rp = reinterpret_cast<const T*>(__shfl_sync(0xffffffffu, my_row, src));
        const bool rok = __shfl_sync(0xffffffffu, (int)row_ok, src) != 0;
        v[k] = make_uint4(0u, 0u, 0u, 0u);
        if (rok && c * 8 < p.Dv) v[k] = *reinterpret_cast<const uint4*>(rp + c * 8);
      }
#pragma unroll
      for (int k = 0; k < 32 / RPI; ++k) {
        const int rr = (warp & 3) * 32 + k * RPI + sub;  // row within the tile
        *reinterpret_cast<uint4*>(qt + (c >> 3) * 16384 + sw128_chunk(rr, c & 7)) = v[k];
      }
    }
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) mbar_arrive(smem_addr(q_ready));

    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    const uint32_t t_s = tmem + (uint32_t)(t * 256) + lane_base;  // S / P buffers of this tile
    const uint32_t t_o = t_s + 128u;                               // O of this tile
    float m_ref = -INFINITY;  // reference max (log2 domain) of this row
    float l = 0.f;
    bool ok = true;
    for (int j = 0; j < n_chunks && tile_on; ++j) {
      const int sb = j & 1;
      if (!mbar_test_then_wait(smem_addr(&s_full[t * 2 + sb]), (uint32_t)((j >> 1) & 1))) {
        ok = false;
        break;
      }
      tmem_fence_after();
      float x[kChunk];  // raw scores q.k of this row's 64 tokens
      {
        uint32_t r0[32], r1[32];
        tmem_ld32(t_s + sb * kChunk, r0);
        tmem_ld32(t_s + sb * kChunk + 32, r1);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          x[i] = __uint_as_float(r0[i]);
          x[32 + i] = __uint_as_float(r1[i]);
        }
      }
      const int tok0 = kv_lo + j * kChunk;
      if (tok0 + kChunk - 1 > lim) {  // causal / end-of-range mask in this chunk
#pragma unroll
        for (int i = 0; i < kChunk; ++i)
          if (tok0 + i > lim) x[i] = -INFINITY;
      }
      float mx_raw = -INFINITY;
#pragma unroll
      for (int i = 0; i < kChunk; ++i) mx_raw = fmaxf(mx_raw, x[i]);
      const float sl2 = p.scale_log2;  // > 0, so max(x * s) = s * max(x)
      const float mx = mx_raw * sl2;
      // reference max: move it (and rescale O) only when the row max grows a lot
      float alpha = 1.f;
      bool move = false;
      if (mx > m_ref + kRescaleThreshold || (m_ref == -INFINITY && mx != -INFINITY)) {
        alpha = (m_ref == -INFINITY) ? 0.f : ex2(m_ref - mx);
        m_ref = mx;
        move = true;
      }
      const float nbase = (m_ref == -INFINITY) ? 0.f : -m_ref;

      // O rescale (warp-collective TMEM load/store) once the PV of chunk j-1 is done
      if (__any_sync(0xffffffffu, move && j > 0)) {
        if (!mbar_wait_bounded(smem_addr(&pv_done[t * 2 + ((j - 1) & 1)]), (uint32_t)(((j - 1) >> 1) & 1))) {
          ok = false;
          break;
        }
        tmem_fence_after();
        const float a = (move && j > 0) ? alpha : 1.f;
#pragma unroll
        for (int c0 = 0; c0 < D; c0 += 32) {
          uint32_t o[32];
          tmem_ld32(t_o + c0, o);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * a);
          tmem_st32(t_o + c0, o);
        }
      }
      // P row over this chunk's S columns: hi at +0..31, lo at +32..63
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
            split_bf16_pair(p0, p1, hi[i], lo[i]);
          } else {
            hi[i] = pack2<T>(p0, p1);
            lo[i] = 0u;
          }
        }
        tmem_st8(t_s + sb * kChunk + piece * 8, hi);
        if (kSplit) tmem_st8(t_s + sb * kChunk + 32 + piece * 8, lo);
      }
      l = l * alpha + ps;
      // tail chunk: V rows at or past kv_end hold stale data; zero them (P is 0
      // there).  Tile 0's warpgroup does it before its P is published; the PV of
      // tile 1 is issued after tile 0's, so it sees the zeros too.
      const int valid = kv_end - tok0;
      if (t == 0 && valid < kChunk) {
        uint8_t* vbase = s_kv + (j % S) * KV_BYTES + HALVES * HALF_BYTES;
        const int nrows = kChunk - valid;
        for (int i = r; i < nrows * HALVES * 8; i += 128) {
          const int row = valid + i / (HALVES * 8);
          const int rem = i % (HALVES * 8);
          *reinterpret_cast<uint4*>(vbase + (rem >> 3) * HALF_BYTES + row * 128 + (rem & 7) * 16) =
              make_uint4(0u, 0u, 0u, 0u);
        }
        fence_proxy_async_smem();
      }
      tmem_wait_st();
      tmem_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_addr(&p_full[t * 2 + sb]));
    }

    // ---- epilogue ----
    if (tile_on && ok && n_chunks > 0) {
      const int jl = n_chunks - 1;
      ok = mbar_wait_bounded(smem_addr(&pv_done[t * 2 + (jl & 1)]), (uint32_t)((jl >> 1) & 1));
    }
    if (!ok && lane == 0) raise_flag(p.status, PA_DEVERR_WAIT_TIMEOUT);
    tmem_fence_after();
    const bool have_o = tile_on && n_chunks > 0;  // warp-uniform
    if constexpr (kPrefix) {
      // (m, l) and the unnormalised O of this row's prefix part, for the decode
      // kernel to fold in; an empty or failed part is (-inf, 0, 0).
      const bool have = ok && l > 0.f;
      const long long ridx = (long long)split * p.B * p.Hq * p.q_len +
                             ((long long)b * p.Hq + h * p.G + g) * p.q_len + tq;
      if (row_ok) p.pre_ml[ridx] = make_float2(have ? m_ref : -INFINITY, have ? l : 0.f);
      float* arow = p.pre_acc + ridx * D;
      // The warp's 32 rows go out through shared memory, whole rows per store
      // instruction.  Staging space: tile 0 the Q tiles, tile 1 the K/V ring.
      // Both are free once this tile's last P.V has completed: its commit
      // tracks every MMA issued before it, and tile 1's last P.V is the last
      // MMA.  Without a clean finish (a wait ran out, copies may still be in
      // flight) the rows go out one per thread.
      const bool staged = tile_on && __all_sync(0xffffffffu, ok) && __any_sync(0xffffffffu, row_ok);
      if (staged) {
        constexpr int CHF = D / 4;  // 16-byte pieces per fp32 row
        uint8_t* sw = (t == 0 ? s_q : s_kv) + (warp & 3) * (32 * D * 4);
#pragma unroll
        for (int c0 = 0; c0 < D; c0 += 32) {
          uint32_t o[32];
          if (have_o) {
            tmem_ld32(t_o + c0, o);
            tmem_wait_ld();
          }
#pragma unroll
          for (int i = 0; i < 32; i += 4) {
            uint4 v = make_uint4(0u, 0u, 0u, 0u);
            if (have) v = make_uint4(o[i], o[i + 1], o[i + 2], o[i + 3]);
            const int piece = (c0 + i) / 4;
            *reinterpret_cast<uint4*>(sw + lane * (D * 4) + ((piece ^ lane) & (CHF - 1)) * 16) = v;
          }
        }
        __syncwarp();
        constexpr int RPI = 32 / CHF;  // rows per store instruction
        const int sub = lane / CHF, pc = lane % CHF;
        const unsigned long long my_row = reinterpret_cast<unsigned long long>(arow);
#pragma unroll 4
        for (int k = 0; k < 32 / RPI; ++k) {
          const int src = k * RPI + sub;
          float* dst = reinterpret_cast<float*>(__shfl_sync(0xffffffffu, my_row, src));
          const bool rok = __shfl_sync(0xffffffffu, (int)row_ok, src) != 0;
          const uint4 v = *reinterpret_cast<const uint4*>(sw + src * (D * 4) + ((pc ^ src) & (CHF - 1)) * 16);
          if (rok) *reinterpret_cast<uint4*>(dst + pc * 4) = v;
        }
      } else {
#pragma unroll
        for (int c0 = 0; c0 < D; c0 += 32) {
          uint32_t o[32];
          if (have_o) {
            tmem_ld32(t_o + c0, o);
            tmem_wait_ld();
          }
          if (row_ok) {
#pragma unroll
            for (int i = 0; i < 32; i += 4) {
              float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
              if (have)
                v = make_float4(__uint_as_float(o[i]), __uint_as_float(o[i + 1]), __uint_as_float(o[i + 2]),
                                __uint_as_float(o[i + 3]));
              *reinterpret_cast<float4*>(arow + c0 + i) = v;
            }
          }
        }
      }
      if (p.splits > 1) {
        // The last split of this CTA's rows to finish merges every split's
        // state of those rows into split 0 (log-sum-exp), so the decode kernel
        // folds one state per row.
        __threadfence();
        asm volatile("bar.sync 1, 256;" ::: "memory");  // the eight softmax warps
        if (tid == 0) s_last = atomicAdd(&p.pre_cnt[tile_id], 1) == p.splits - 1;
        asm volatile("bar.sync 1, 256;" ::: "memory");
        if (s_last && row_ok) {
          __threadfence();
          const long long R = (long long)p.B * p.Hq * p.q_len;
          const long long r0 = ridx - (long long)split * R;  // this row in split 0
          float M = -INFINITY;
          for (int sp = 0; sp < p.splits; ++sp) M = fmaxf(M, __ldcg(&p.pre_ml[sp * R + r0]).x);
          const float base = (M == -INFINITY) ? 0.f : M;
          float lsum = 0.f;
          for (int sp = 0; sp < p.splits; ++sp) {
            const float2 ml = __ldcg(&p.pre_ml[sp * R + r0]);
            lsum += ex2(ml.x - base) * ml.y;
          }
          for (int c0 = 0; c0 < D; c0 += 32) {
            float4 a[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) a[i] = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int sp = 0; sp < p.splits; ++sp) {
              const float w = ex2(__ldcg(&p.pre_ml[sp * R + r0]).x - base);
              const float4* src = reinterpret_cast<const float4*>(p.pre_acc + (sp * R + r0) * D + c0);
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                const float4 v = __ldcg(src + i);
                a[i].x = fmaf(w, v.x, a[i].x);
                a[i].y = fmaf(w, v.y, a[i].y);
                a[i].z = fmaf(w, v.z, a[i].z);
                a[i].w = fmaf(w, v.w, a[i].w);
              }
            }
            float4* dst = reinterpret_cast<float4*>(p.pre_acc + r0 * D + c0);
#pragma unroll
            for (int i = 0; i < 8; ++i) dst[i] = a[i];
          }
          p.pre_ml[r0] = make_float2(M, lsum);
        }
      }
    } else {
      T* orow = static_cast<T*>(p.out) + (long long)b * p.o_sb + (long long)(h * p.G + g) * p.o_sh +
                (long long)tq * p.o_st;
      const float inv = (ok && l > 0.f) ? 1.f / l : 0.f;
      // As in the prefix epilogue: the warp's rows go out through shared
      // memory (this tile's Q tile, free once its last P.V has completed),
      // whole rows per store instruction.
      const bool staged = tile_on && __all_sync(0xffffffffu, ok) && __any_sync(0xffffffffu, row_ok);
      if (staged) {
        constexpr int CHB = D / 8;  // 16-byte pieces per output row
        uint8_t* sw = s_q + t * QT_BYTES + (warp & 3) * (32 * D * 2);
#pragma unroll
        for (int c0 = 0; c0 < D; c0 += 32) {
          uint32_t o[32];
          if (have_o) {
            tmem_ld32(t_o + c0, o);
            tmem_wait_ld();
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = 0u;
          }
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            uint4 v;
            v.x = pack2<T>(__uint_as_float(o[i]) * inv, __uint_as_float(o[i + 1]) * inv);
            v.y = pack2<T>(__uint_as_float(o[i + 2]) * inv, __uint_as_float(o[i + 3]) * inv);
            v.z = pack2<T>(__uint_as_float(o[i + 4]) * inv, __uint_as_float(o[i + 5]) * inv);
            v.w = pack2<T>(__uint_as_float(o[i + 6]) * inv, __uint_as_float(o[i + 7]) * inv);
            const int piece = (c0 + i) / 8;
            *reinterpret_cast<uint4*>(sw + lane * (D * 2) + ((piece ^ lane) & (CHB - 1)) * 16) = v;
          }
        }
        __syncwarp();
        constexpr int RPI = 32 / CHB;  // rows per store instruction
        const int sub = lane / CHB, pc = lane % CHB;
        const unsigned long long my_row = reinterpret_cast<unsigned long long>(orow);
#pragma unroll 4
        for (int k = 0; k < 32 / RPI; ++k) {
          const int src = k * RPI + sub;
          T* dst = reinterpret_cast<T*>(__shfl_sync(0xffffffffu, my_row, src));
          const bool rok = __shfl_sync(0xffffffffu, (int)row_ok, src) != 0;
          const uint4 v = *reinterpret_cast<const uint4*>(sw + src * (D * 2) + ((pc ^ src) & (CHB - 1)) * 16);
          if (rok && pc * 8 < p.Dv) *reinterpret_cast<uint4*>(dst + pc * 8) = v;
        }
      } else {
#pragma unroll
        for (int c0 = 0; c0 < D; c0 += 32) {
          uint32_t o[32];
          if (have_o) {
            tmem_ld32(t_o + c0, o);
            tmem_wait_ld();
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = 0u;
          }
          if (row_ok) {
#pragma unroll
            for (int i = 0; i < 32; i += 8) {
              if (c0 + i >= p.Dv) break;  // columns past the head_dim
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
    }
  }

  tmem_fence_before();
  __syncthreads();
  if (warp == 0) {
    tmem_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

size_t prefill_umma_smem_bytes(int D) {
  const size_t halves = (size_t)D / 64;
  const size_t stages = D == 128 ? kUmmaStages<128>::value : kUmmaStages<64>::value;
  return 1024 + stages * 2 * halves * kChunk * 128 + 2 * halves * 128 * 128 + 256;
}

template <typename T, int D, bool kPrefix>
static cudaError_t launch_umma_impl(const DecodeParams& p, const CUtensorMap& tmk, const CUtensorMap& tmv, bool pdl,
                                    cudaStream_t stream) {
  const size_t smem = prefill_umma_smem_bytes(D);
  static bool prepared[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !prepared[dev]) {
    cudaError_t e = cudaFuncSetAttribute(prefill_umma_kernel<T, D, kPrefix>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    prepared[dev] = true;
  }
  const long long ctas =
      kPrefix ? (long long)p.splits * p.num_groups * p.Hkv * (((long long)p.max_members * p.GQ + kTileRows - 1) / kTileRows)
              : (long long)p.B * p.Hkv * ((p.GQ + kTileRows - 1) / kTileRows);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)ctas);
  cfg.blockDim = dim3(umma_threads(kPrefix));
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = pdl ? attr : nullptr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, prefill_umma_kernel<T, D, kPrefix>, tmk, tmv, p);
}

template <bool kPrefix>
static cudaError_t launch_umma(const DecodeParams& p, const CUtensorMap& tmk, const CUtensorMap& tmv, int dtype,
                               bool pdl, cudaStream_t stream) {
  if (dtype == PA_DTYPE_BFLOAT16) {
    if (p.D == 128) return launch_umma_impl<__nv_bfloat16, 128, kPrefix>(p, tmk, tmv, pdl, stream);
    if (p.D == 64) return launch_umma_impl<__nv_bfloat16, 64, kPrefix>(p, tmk, tmv, pdl, stream);
  } else if (dtype == PA_DTYPE_FLOAT16) {
    if (p.D == 128) return launch_umma_impl<__half, 128, kPrefix>(p, tmk, tmv, pdl, stream);
    if (p.D == 64) return launch_umma_impl<__half, 64, kPrefix>(p, tmk, tmv, pdl, stream);
  }
  return cudaErrorInvalidValue;
}

cudaError_t launch_prefill_umma(const DecodeParams& p, const CUtensorMap& tmk, const CUtensorMap& tmv, int dtype,
                                bool pdl, cudaStream_t stream) {
  return launch_umma<false>(p, tmk, tmv, dtype, pdl, stream);
}

cudaError_t launch_prefix_umma(const DecodeParams& p, const CUtensorMap& tmk, const CUtensorMap& tmv, int dtype,
                               bool pdl, cudaStream_t stream) {
  return launch_umma<true>(p, tmk, tmv, dtype, pdl, stream);
}

}  // namespace pa
