// pa_decode_f32.cu — paged decode attention for fp32 caches (CUDA cores).
//
// fp32 must match the reference to 1e-5, so it stays off the tensor cores
// (TF32 would not).  The kernel follows the reference's per-row CPU algorithm
// block by block (runtime/phase2/paged_attention_triton.py:663-704):
//   for each cache block: scores = (q . k) * scale over the block's tokens,
//   m_new = max(m, max(scores)), p = exp(scores - m_new), alpha = exp(m - m_new),
//   l = l * alpha + sum(p), acc = acc * alpha + p @ v;   out = acc / l
// with a causal limit for query token t of L - q_len + t.
// One CTA serves one (sequence, kv head); each warp takes query rows of the GQA
// group in turn; a lane scores one token of the block and owns D/32 output dims.
// The fp32 configurations are small (launch-bound), so this kernel favours a
// direct restatement over bandwidth tricks.
#include <math.h>

#include "pa_common.cuh"
#include "pa_internal.h"

namespace pa {

template <int DPL>  // head_dim / 32
__global__ void __launch_bounds__(128) decode_f32_kernel(const DecodeParams p) {
  constexpr int D = DPL * 32;
  constexpr int kWarps = 4;
  __shared__ float s_q[kWarps][D];

  pdl_wait_previous();

  const int b = blockIdx.x / p.Hkv;
  const int h = blockIdx.x - b * p.Hkv;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  int L = p.context_lens[b] + p.len_offset;
  const int cap = p.max_blocks * p.bs;
  if (L > cap) {
    if (threadIdx.x == 0 && h == 0) raise_flag(p.status, PA_DEVERR_TABLE_UNDERRUN);
    L = cap;
  }
  if (L < 0) L = 0;

  const float* kc = static_cast<const float*>(p.k_cache);
  const float* vc = static_cast<const float*>(p.v_cache);

  for (int qr = warp; qr < p.GQ; qr += kWarps) {
    const int g = qr / p.q_len;
    const int t = qr - g * p.q_len;
    const int head = h * p.G + g;
    const float* qp = static_cast<const float*>(p.q) + (long long)b * p.q_sb +
                      (long long)head * p.q_sh + (long long)t * p.q_st;
#pragma unroll
    for (int k = 0; k < DPL; ++k) s_q[warp][lane + 32 * k] = qp[lane + 32 * k];
    __syncwarp();

    int ntok = L - p.q_len + t + 1;  // tokens 0 .. L - q_len + t
    if (ntok > L) ntok = L;
    if (ntok < 0) ntok = 0;

    float m = -INFINITY, l = 0.f;
    float acc[DPL];
#pragma unroll
    for (int k = 0; k < DPL; ++k) acc[k] = 0.f;

    for (int blk = 0; blk * p.bs < ntok; ++blk) {
      const int phys = p.block_tables[(long long)b * p.bt_stride + blk];
      if (phys < 0 || phys >= p.num_blocks) {
        if (lane == 0) raise_flag(p.status, PA_DEVERR_BLOCK_ID_RANGE);
        continue;
      }
      const int take = min(p.bs, ntok - blk * p.bs);
      const float* kb = kc + (long long)phys * p.k_sblk + (long long)h * p.k_sh;
      const float* vb = vc + (long long)phys * p.v_sblk + (long long)h * p.v_sh;
      for (int c0 = 0; c0 < take; c0 += 32) {
        const int cnt = min(32, take - c0);
        float sc = -INFINITY;
        if (lane < cnt) {
          const float* kr = kb + (long long)(c0 + lane) * p.k_st;
          float dot = 0.f;
#pragma unroll 8
          for (int d = 0; d < D; ++d) dot = fmaf(s_q[warp][d], kr[d], dot);
          sc = dot * p.scale;
        }
        float bm = sc;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, o));
        const float m_new = fmaxf(m, bm);
        const float alpha = (m == -INFINITY) ? 0.f : expf(m - m_new);
        const float pl = (lane < cnt) ? expf(sc - m_new) : 0.f;
        float ps = pl;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
        l = l * alpha + ps;
#pragma unroll
        for (int k = 0; k < DPL; ++k) acc[k] *= alpha;
        for (int tt = 0; tt < cnt; ++tt) {
          const float pt = __shfl_sync(0xffffffffu, pl, tt);
          const float* vr = vb + (long long)(c0 + tt) * p.v_st;
#pragma unroll
          for (int k = 0; k < DPL; ++k) acc[k] = fmaf(pt, vr[lane + 32 * k], acc[k]);
        }
        m = m_new;
      }
    }

    float* op = static_cast<float*>(p.out) + (long long)b * p.o_sb + (long long)head * p.o_sh +
                (long long)t * p.o_st;
    const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll
    for (int k = 0; k < DPL; ++k) op[lane + 32 * k] = acc[k] * inv;
    __syncwarp();
  }
}

cudaError_t launch_decode_f32(const DecodeParams& p, bool pdl, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(p.B * p.Hkv));
  cfg.blockDim = dim3(128);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = pdl ? attr : nullptr;
  cfg.numAttrs = pdl ? 1 : 0;
  switch (p.D) {
    case 32:
      return cudaLaunchKernelEx(&cfg, decode_f32_kernel<1>, p);
    case 64:
      return cudaLaunchKernelEx(&cfg, decode_f32_kernel<2>, p);
    case 128:
      return cudaLaunchKernelEx(&cfg, decode_f32_kernel<4>, p);
    case 256:
      return cudaLaunchKernelEx(&cfg, decode_f32_kernel<8>, p);
    default:
      return cudaErrorInvalidValue;
  }
}

}  // namespace pa
