// pa_prefill_mma.cu — multi-query attention over paged KV (chunked prefill,
// long speculative verification), fp16 / bf16, sm_100a.
//
// Same math and row layout as the decode kernel (token-major rows of one KV
// head, causal limit L - q_len + t per query token; pa_tile_math.cuh), but
// built for many query rows per KV head: a CTA owns a 128-row tile of one
// (sequence, kv head) — 8 consumer warps x 16 rows — and a producer warp
// streams the sequence's 16-token K/V units by TMA into a 6-stage shared ring
// (full / empty mbarriers, every wait bounded).  Each K/V tile is read once per
// 128 query rows instead of once per 16, and the tile stops at its latest
// row's causal limit.  Tiles of the latest query tokens (the most work) are
// scheduled first.  No split, so no partials: every warp stores its own rows.
#include <math.h>

#include "pa_common.cuh"
#include "pa_internal.h"
#include "pa_tile_math.cuh"

namespace pa {

template <typename T, int D>
__global__ void __launch_bounds__(kPrefillThreads, 1)
    prefill_mma_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
                       const DecodeParams p) {
  constexpr int HALVES = D / 64;
  constexpr uint32_t TILE_BYTES = 16 * D * 2;
  constexpr uint32_t STAGE_BYTES = 2 * TILE_BYTES;
  constexpr int S = kPrefillStages;

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_addr(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  const uint32_t ring = smem_addr(smem);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)S * STAGE_BYTES);
  uint64_t* empty = full + S;

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int MT = (p.GQ + 127) / 128;
  // The tiles of one (sequence, kv head) read the same K/V: adjacent block
  // indices run them in the same wave, so all but the first read hit L2.
  // Within a (sequence, kv head), the latest (heaviest) tiles first.
  const int mt = MT - 1 - (int)(blockIdx.x % MT);
  const int bh = (int)(blockIdx.x / MT);
  const int b = bh / p.Hkv;
  const int h = bh - b * p.Hkv;

  int L = p.context_lens[b] + p.len_offset;
  const int cap = p.max_blocks * p.bs;
  if (L > cap) {
    if (tid == 0 && h == 0 && mt == MT - 1) raise_flag(p.status, PA_DEVERR_TABLE_UNDERRUN);
    L = cap;
  }
  if (L < 0) L = 0;
  const int row0 = mt * 128;
  const int rows_tile = min(128, p.GQ - row0);
  const int active = (rows_tile + 15) / 16;  // consumer warps that own rows
  const int lim_tile = L - p.q_len + (row0 + rows_tile - 1) / p.G;
  const int n_units = lim_tile < 0 ? 0 : (lim_tile + kUnitTokens) / kUnitTokens;

  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(smem_addr(&full[s]), 1);
      mbar_init(smem_addr(&empty[s]), active);
    }
    prefetch_tensormap(&tmk);
    prefetch_tensormap(&tmv);
  }
  fence_mbar_init();
  __syncthreads();
  pdl_wait_previous();

  if (warp == kPrefillWarps) {
    // ---- producer warp: lane 0 issues, the warp shares the block-table window ----
    int win_base = -1, win_val = -1;
    const int bs = p.bs;
    for (int u = 0; u < n_units; ++u) {
      const int slot = u % S;
      const int k = u / S;
      if (k > 0) {
        int ok = 1;
        if (lane == 0) ok = mbar_wait_bounded(smem_addr(&empty[slot]), (uint32_t)((k - 1) & 1)) ? 1 : 0;
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) {
          if (lane == 0) raise_flag(p.status, PA_DEVERR_WAIT_TIMEOUT);
          return;
        }
      }
      const int tok0 = u * kUnitTokens;
      const int lb0 = tok0 / bs;
      const int need = bs >= kUnitTokens ? 1 : kUnitTokens / bs;
      if (win_base < 0 || lb0 < win_base || lb0 + need > win_base + 32) {
        win_base = lb0;
        const int e = lb0 + lane;
        win_val = (e < p.max_blocks) ? __ldg(&p.block_tables[(long long)b * p.bt_stride + e]) : -1;
      }
      const int phys0 = __shfl_sync(0xffffffffu, win_val, lb0 - win_base);
      const int phys1 = __shfl_sync(0xffffffffu, win_val, (lb0 + 1 - win_base) & 31);
      // One box per lane (K or V x 64-column half, x block for size 8), in one
      // instruction: a thread's bulk-tensor copies issue one after another.
      const uint32_t stage = ring + (uint32_t)slot * STAGE_BYTES;
      const uint32_t bar = smem_addr(&full[slot]);
      const bool need1 = bs < kUnitTokens && (lb0 + 1) * bs < L;
      const uint32_t box_bytes = bs >= kUnitTokens ? 2048u : (uint32_t)bs * 128u;
      const int nbox = (need1 ? 2 : 1) * HALVES * 2;
      if (lane == 0) {
        if (phys0 < 0 || phys0 >= p.num_blocks || (need1 && (phys1 < 0 || phys1 >= p.num_blocks)))
          raise_flag(p.status, PA_DEVERR_BLOCK_ID_RANGE);
        mbar_arrive_expect_tx(bar, (uint32_t)nbox * box_bytes);
      }
      __syncwarp();
      if (lane < nbox) {  // lane -> (block j, K or V, half)
        const int j = lane / (2 * HALVES), kv = (lane / HALVES) & 1, hf = lane % HALVES;
        const int y = bs >= kUnitTokens ? tok0 - lb0 * bs : 0;
        tma_load_4d(stage + (uint32_t)kv * TILE_BYTES + (uint32_t)hf * 2048u + (uint32_t)j * box_bytes,
                    kv ? &tmv : &tmk, bar, hf * 64, y, h, j ? phys1 : phys0);
      }
      __syncwarp();
    }
    return;
  }
  if (warp >= active) return;  // no rows for this warp (the empty barriers count active warps only)

  // ---- consumer warp: 16 query rows ----
  const int quad = lane & 3;
  const int qrow0 = lane >> 2;
  const int qr0 = row0 + warp * 16 + qrow0;
  const int qr1 = qr0 + 8;
  const T* qp0 = nullptr;
  const T* qp1 = nullptr;
  T* op0 = nullptr;
  T* op1 = nullptr;
  int lim0 = L - 1, lim1 = L - 1;
  if (qr0 < p.GQ) {
    const int t = qr0 / p.G, g = qr0 - (qr0 / p.G) * p.G;
    const long long hq = (long long)(h * p.G + g);
    qp0 = static_cast<const T*>(p.q) + (long long)b * p.q_sb + hq * p.q_sh + (long long)t * p.q_st;
    op0 = static_cast<T*>(p.out) + (long long)b * p.o_sb + hq * p.o_sh + (long long)t * p.o_st;
    lim0 = L - p.q_len + t;
  }
  if (qr1 < p.GQ) {
    const int t = qr1 / p.G, g = qr1 - (qr1 / p.G) * p.G;
    const long long hq = (long long)(h * p.G + g);
    qp1 = static_cast<const T*>(p.q) + (long long)b * p.q_sb + hq * p.q_sh + (long long)t * p.q_st;
    op1 = static_cast<T*>(p.out) + (long long)b * p.o_sb + hq * p.o_sh + (long long)t * p.o_st;
    lim1 = L - p.q_len + t;
  }
  const int wlast = min(row0 + warp * 16 + 15, p.GQ - 1);
  const int lim_w = L - p.q_len + wlast / p.G;
  const int n_w = lim_w < 0 ? 0 : (lim_w + kUnitTokens) / kUnitTokens;  // units this warp needs
  const int mask_from = L - p.q_len + (row0 + warp * 16) / p.G;

  uint32_t qa[D / 16][4];
  load_query_frags<T, D>(qa, qp0, qp1, quad, p.Dv);
  float o_acc[D / 8][4];
#pragma unroll
  for (int nd = 0; nd < D / 8; ++nd) o_acc[nd][0] = o_acc[nd][1] = o_acc[nd][2] = o_acc[nd][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;

  for (int u = 0; u < n_units; ++u) {
    const int slot = u % S;
    const uint32_t bar = smem_addr(&full[slot]);
    if (!mbar_wait_bounded(bar, (uint32_t)((u / S) & 1))) {
      if (lane == 0) raise_flag(p.status, PA_DEVERR_WAIT_TIMEOUT);
      return;  // the producer's own bounded waits end it
    }
    if (u < n_w) {
      const uint32_t kbase = ring + (uint32_t)slot * STAGE_BYTES;
      attend_unit<T, D>(kbase, kbase + TILE_BYTES, qa, o_acc, m0, m1, l0, l1, u * kUnitTokens, L, lim0, lim1,
                        mask_from, p.scale_log2, lane);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(smem_addr(&empty[slot]));
  }

  float lt0 = l0 + __shfl_xor_sync(0xffffffffu, l0, 1);
  float lt1 = l1 + __shfl_xor_sync(0xffffffffu, l1, 1);
  lt0 += __shfl_xor_sync(0xffffffffu, lt0, 2);
  lt1 += __shfl_xor_sync(0xffffffffu, lt1, 2);
  store_rows<T, D>(op0, op1, o_acc, lt0, lt1, quad, p.Dv);
}

size_t prefill_smem_bytes(int D) {
  return 1024 + (size_t)kPrefillStages * (2u * 16u * (size_t)D * 2u) + 2 * kPrefillStages * 8;
}

template <typename T, int D>
static cudaError_t launch_prefill_impl(const DecodeParams& p, const CUtensorMap& tmk, const CUtensorMap& tmv,
                                       bool pdl, cudaStream_t stream) {
  const size_t smem = prefill_smem_bytes(D);
  static bool prepared[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !prepared[dev]) {
    cudaError_t e = cudaFuncSetAttribute(prefill_mma_kernel<T, D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) return e;
    prepared[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)((long long)p.B * p.Hkv * ((p.GQ + 127) / 128)));
  cfg.blockDim = dim3(kPrefillThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = pdl ? attr : nullptr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, prefill_mma_kernel<T, D>, tmk, tmv, p);
}

cudaError_t launch_prefill_mma(const DecodeParams& p, const CUtensorMap& tmk, const CUtensorMap& tmv, int dtype,
                               bool pdl, cudaStream_t stream) {
  if (dtype == PA_DTYPE_BFLOAT16) {
    if (p.D == 128) return launch_prefill_impl<__nv_bfloat16, 128>(p, tmk, tmv, pdl, stream);
    if (p.D == 64) return launch_prefill_impl<__nv_bfloat16, 64>(p, tmk, tmv, pdl, stream);
  } else if (dtype == PA_DTYPE_FLOAT16) {
    if (p.D == 128) return launch_prefill_impl<__half, 128>(p, tmk, tmv, pdl, stream);
    if (p.D == 64) return launch_prefill_impl<__half, 64>(p, tmk, tmv, pdl, stream);
  }
  return cudaErrorInvalidValue;
}

}  // namespace pa
