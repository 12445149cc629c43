// pa_decode_f32.cu — paged decode attention for fp32 caches (CUDA cores).
//
// fp32 must match the reference to 1e-5, so it stays off the tensor cores
// (TF32 would not).  The math is the reference's per-row CPU algorithm
// (runtime/phase2/paged_attention_triton.py:663-704), applied to chunks of at
// most 16 tokens of one cache block:
//   scores = (q . k) * scale,  m_new = max(m, max(scores)),
//   p = exp(scores - m_new),   alpha = exp(m - m_new),
//   l = l * alpha + sum(p),    acc = acc * alpha + p @ v;      out = acc / l
// with the causal limit L - q_len + t for query token t.
//
// One CTA serves one (sequence, kv head).  Its warps take the sequence's
// blocks in turn (block w, w + NW, ...), each keeping (m, l, acc) for every
// query row of the GQA group (up to 16 rows per pass); a chunk's K and V are
// staged in shared memory with a padded row pitch (D + 1 floats, so lanes
// reading different tokens hit different banks).  Lanes score one token each
// for all rows, then own D/32 output dims for the P.V update.  At the end the
// warps' states are merged with the log-sum-exp rule.  The fp32 configurations
// are small, so this kernel aims at latency: many warps in flight per row.
#include <math.h>

#include "pa_common.cuh"
#include "pa_internal.h"

namespace pa {

namespace {
constexpr int kF32Warps = 8;
constexpr int kF32Chunk = 16;  // tokens per staged chunk
}  // namespace

// DPL = head_dim / 32; kF32Rows = query rows handled per pass (4, 8 or 16,
// the smallest that holds the GQA group's G * q_len rows).
template <int DPL, int kF32Rows>
__global__ void __launch_bounds__(kF32Warps * 32) decode_f32_kernel(const DecodeParams p) {
  constexpr int D = DPL * 32;
  constexpr int PITCH = D + 1;
  extern __shared__ float f32_smem[];
  // [rows][D] queries | (m, l) per warp and row | per warp: K chunk, V chunk
  // [kF32Chunk][PITCH] and P [rows][kF32Chunk].  After its last block a warp
  // reuses its own K/V chunk area for its [rows][D] accumulator.
  constexpr int kWarpFloats = 2 * kF32Chunk * PITCH + kF32Rows * kF32Chunk;
  static_assert(kF32Rows * D <= 2 * kF32Chunk * PITCH, "accumulator must fit the staging area");
  static_assert(kF32Rows <= 32, "one lane per row in the merge bookkeeping");
  float* s_q = f32_smem;
  float* s_ml = s_q + kF32Rows * D;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  float* s_k = s_ml + kF32Warps * 2 * kF32Rows + warp * kWarpFloats;
  float* s_v = s_k + kF32Chunk * PITCH;
  float* s_p = s_v + kF32Chunk * PITCH;

  pdl_wait_previous();

  const int b = blockIdx.x / p.Hkv;
  const int h = blockIdx.x - b * p.Hkv;

  int L = p.context_lens[b] + p.len_offset;
  const int cap = p.max_blocks * p.bs;
  if (L > cap) {
    if (threadIdx.x == 0 && h == 0) raise_flag(p.status, PA_DEVERR_TABLE_UNDERRUN);
    L = cap;
  }
  if (L < 0) L = 0;
  const int first_limit = L - p.q_len;  // last token row t=0 may attend
  const int ntok_max = L;               // tokens any row may attend
  const int nblk = (ntok_max + p.bs - 1) / p.bs;

  const float* kc = static_cast<const float*>(p.k_cache);
  const float* vc = static_cast<const float*>(p.v_cache);

  for (int r0 = 0; r0 < p.GQ; r0 += kF32Rows) {
    const int R = min(kF32Rows, p.GQ - r0);
    __syncthreads();  // previous pass's merge area and queries are free
    for (int i = threadIdx.x; i < R * D; i += blockDim.x) {
      const int r = i / D, d = i - (i / D) * D;
      const int qr = r0 + r;
      const int g = qr / p.q_len, t = qr - (qr / p.q_len) * p.q_len;
      s_q[r * D + d] = d < p.Dv ? static_cast<const float*>(p.q)[(long long)b * p.q_sb +
                                                                  (long long)(h * p.G + g) * p.q_sh +
                                                                  (long long)t * p.q_st + d]
                                : 0.f;
    }
    __syncthreads();

    float m[kF32Rows], l[kF32Rows], acc[kF32Rows][DPL];
#pragma unroll
    for (int r = 0; r < kF32Rows; ++r) {
      m[r] = -INFINITY;
      l[r] = 0.f;
#pragma unroll
      for (int j = 0; j < DPL; ++j) acc[r][j] = 0.f;
    }

    for (int blk = warp; blk < nblk; blk += kF32Warps) {
      const int phys = p.block_tables[(long long)b * p.bt_stride + blk];
      if (phys < 0 || phys >= p.num_blocks) {
        if (lane == 0) raise_flag(p.status, PA_DEVERR_BLOCK_ID_RANGE);
        continue;
      }
      const int take = min(p.bs, ntok_max - blk * p.bs);
      const float* kb = kc + (long long)phys * p.k_sblk + (long long)h * p.k_sh;
      const float* vb = vc + (long long)phys * p.v_sblk + (long long)h * p.v_sh;
      for (int c0 = 0; c0 < take; c0 += kF32Chunk) {
        const int cnt = min(kF32Chunk, take - c0);
        const int tok0 = blk * p.bs + c0;  // absolute position of the chunk's first token
        if (tok0 > first_limit + p.q_len - 1) break;  // no row attends past L - 1
        __syncwarp();
        // Stage the chunk: every copy of the chunk is in flight at once.
#pragma unroll 4
        for (int t = 0; t < cnt; ++t) {
#pragma unroll
          for (int j = 0; j < DPL; ++j) {
            if (lane + 32 * j >= p.Dv) break;  // no read past the row; those columns are never used
            cp_async_4(smem_addr(&s_k[t * PITCH + lane + 32 * j]), kb + (long long)(c0 + t) * p.k_st + lane + 32 * j);
            cp_async_4(smem_addr(&s_v[t * PITCH + lane + 32 * j]), vb + (long long)(c0 + t) * p.v_st + lane + 32 * j);
          }
        }
        cp_async_wait_all();
        __syncwarp();
        // scores: lane t scores token t for every row
        float sc[kF32Rows];
#pragma unroll
        for (int r = 0; r < kF32Rows; ++r) sc[r] = 0.f;
        if (lane < cnt) {
          const float* kr = s_k + lane * PITCH;
#pragma unroll 4
          for (int d = 0; d < p.Dv; ++d) {
            const float kd = kr[d];
#pragma unroll
            for (int r = 0; r < kF32Rows; ++r)
              if (r < R) sc[r] = fmaf(s_q[r * D + d], kd, sc[r]);
          }
        }
#pragma unroll
        for (int r = 0; r < kF32Rows; ++r) {
          if (r >= R) break;
          const int qr = r0 + r;
          const int t_q = qr - (qr / p.q_len) * p.q_len;
          const int lim = first_limit + t_q;  // last attendable position of this row
          const bool valid = lane < cnt && tok0 + lane <= lim;
          float s = valid ? sc[r] * p.scale : -INFINITY;
          float bm = s;
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, o));
          if (bm == -INFINITY) {  // nothing attendable for this row in this chunk
            if (lane < kF32Chunk) s_p[r * kF32Chunk + lane] = 0.f;
            continue;
          }
          const float m_new = fmaxf(m[r], bm);
          const float alpha = (m[r] == -INFINITY) ? 0.f : expf(m[r] - m_new);
          const float pv = valid ? expf(s - m_new) : 0.f;
          float ps = pv;
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
          l[r] = l[r] * alpha + ps;
          m[r] = m_new;
#pragma unroll
          for (int j = 0; j < DPL; ++j) acc[r][j] *= alpha;
          if (lane < kF32Chunk) s_p[r * kF32Chunk + lane] = pv;
        }
        __syncwarp();
        // acc += P V over the chunk's tokens
        for (int t = 0; t < cnt; ++t) {
          float vd[DPL];
#pragma unroll
          for (int j = 0; j < DPL; ++j) vd[j] = s_v[t * PITCH + lane + 32 * j];
#pragma unroll
          for (int r = 0; r < kF32Rows; ++r) {
            if (r < R) {
              const float pt = s_p[r * kF32Chunk + t];
#pragma unroll
              for (int j = 0; j < DPL; ++j) acc[r][j] = fmaf(pt, vd[j], acc[r][j]);
            }
          }
        }
      }
    }

    // ---- merge the warps' states (log-sum-exp) and store ----
    __syncwarp();
#pragma unroll
    for (int r = 0; r < kF32Rows; ++r) {
      if (r < R) {
        if (lane == 0) {
          s_ml[(warp * 2) * kF32Rows + r] = m[r];
          s_ml[(warp * 2 + 1) * kF32Rows + r] = l[r];
        }
#pragma unroll
        for (int j = 0; j < DPL; ++j) s_k[r * D + lane + 32 * j] = acc[r][j];
      }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < R * D; i += blockDim.x) {
      const int r = i / D, d = i - (i / D) * D;
      if (d >= p.Dv) continue;  // columns past the head_dim
      float M = -INFINITY;
      for (int w = 0; w < kF32Warps; ++w) M = fmaxf(M, s_ml[(w * 2) * kF32Rows + r]);
      float lsum = 0.f, a = 0.f;
      if (M != -INFINITY) {
        for (int w = 0; w < kF32Warps; ++w) {
          const float mw = s_ml[(w * 2) * kF32Rows + r];
          const float sc_w = (mw == -INFINITY) ? 0.f : expf(mw - M);
          lsum += sc_w * s_ml[(w * 2 + 1) * kF32Rows + r];
          a += sc_w * s_ml[kF32Warps * 2 * kF32Rows + w * kWarpFloats + r * D + d];
        }
      }
      const int qr = r0 + r;
      const int g = qr / p.q_len, t = qr - (qr / p.q_len) * p.q_len;
      static_cast<float*>(p.out)[(long long)b * p.o_sb + (long long)(h * p.G + g) * p.o_sh + (long long)t * p.o_st +
                                 d] = lsum > 0.f ? a / lsum : 0.f;
    }
  }
}

static size_t f32_smem_bytes(int D, int kF32Rows) {
  const int pitch = D + 1;
  return sizeof(float) * ((size_t)kF32Rows * D + (size_t)kF32Warps * 2 * kF32Rows +
                          (size_t)kF32Warps * (2 * kF32Chunk * pitch + kF32Rows * kF32Chunk));
}

template <int DPL, int ROWS>
static cudaError_t launch_f32_impl(const DecodeParams& p, bool pdl, cudaStream_t stream) {
  const size_t smem = f32_smem_bytes(DPL * 32, ROWS);
  static bool prepared[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !prepared[dev]) {
    cudaError_t e = cudaFuncSetAttribute(decode_f32_kernel<DPL, ROWS>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    prepared[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(p.B * p.Hkv));
  cfg.blockDim = dim3(kF32Warps * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = pdl ? attr : nullptr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, decode_f32_kernel<DPL, ROWS>, p);
}

template <int DPL>
static cudaError_t launch_f32_rows(const DecodeParams& p, bool pdl, cudaStream_t stream) {
  if (p.GQ <= 4) return launch_f32_impl<DPL, 4>(p, pdl, stream);
  if (p.GQ <= 8) return launch_f32_impl<DPL, 8>(p, pdl, stream);
  return launch_f32_impl<DPL, 16>(p, pdl, stream);
}

cudaError_t launch_decode_f32(const DecodeParams& p, bool pdl, cudaStream_t stream) {
  switch (p.D) {
    case 32:
      return launch_f32_rows<1>(p, pdl, stream);
    case 64:
      return launch_f32_rows<2>(p, pdl, stream);
    case 128:
      return launch_f32_rows<4>(p, pdl, stream);
    default:
      return cudaErrorInvalidValue;
  }
}

}  // namespace pa
