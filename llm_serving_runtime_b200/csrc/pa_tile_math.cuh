// pa_tile_math.cuh — one warp's attention over one 16-token unit, on tensor cores.
//
// Shared by the decode and prefill kernels so both compute exactly the same
// arithmetic.  A warp owns 16 query rows (the A operand of m16n8k16, loaded
// once per row group) and an online-softmax state in the MMA accumulator
// layout: thread (lane) holds rows lane/4 and lane/4 + 8, columns 2*(lane%4),
// +1 of every 8-wide n-tile.  A unit's K and V tiles sit in shared memory as
// TMA wrote them: per 64-element column half, 16 rows of 128 bytes with the
// 128-byte swizzle (16-byte chunk c of row r stored at chunk c ^ (r % 8)).
#pragma once

#include "pa_common.cuh"
#include "pa_internal.h"

namespace pa {

// Tokens of prefix group gi that the cascade's prefix kernel attends: the
// group's prefix length within the host bound and the block-table capacity,
// rounded down to whole 16-token units (the rest is attended per member).
__device__ __forceinline__ int cascade_prefix_tokens(const DecodeParams& p, int gi) {
  const int P = min(max(p.group_prefix[gi], 0), min(p.max_prefix, p.max_blocks * p.bs));
  return P & ~(kUnitTokens - 1);
}


// Whether P is carried as hi + lo parts in the P.V product (bf16 only).
template <typename T>
struct kSplitProbabilities {
  static constexpr bool value = false;
};
template <>
struct kSplitProbabilities<__nv_bfloat16> {
  static constexpr bool value = true;
};

// The two 16-bit halves of a packed register, widened to fp32 exactly.
template <typename T>
__device__ __forceinline__ float lo_half(uint32_t v);
template <typename T>
__device__ __forceinline__ float hi_half(uint32_t v);
template <>
__device__ __forceinline__ float lo_half<__nv_bfloat16>(uint32_t v) {
  return __uint_as_float(v << 16);
}
template <>
__device__ __forceinline__ float hi_half<__nv_bfloat16>(uint32_t v) {
  return __uint_as_float(v & 0xffff0000u);
}
template <>
__device__ __forceinline__ float lo_half<__half>(uint32_t v) {
  return __half2float(__ushort_as_half((unsigned short)(v & 0xffffu)));
}
template <>
__device__ __forceinline__ float hi_half<__half>(uint32_t v) {
  return __half2float(__ushort_as_half((unsigned short)(v >> 16)));
}

// Query fragments (A operand) of the warp's 16 rows; a null row pointer gives
// a zero (padding) row, and columns at or past the head_dim Dv (a multiple of
// 8, <= D) are zero.
template <typename T, int D>
__device__ __forceinline__ void load_query_frags(uint32_t (&qa)[D / 16][4], const T* qp0, const T* qp1,
                                                 int quad, int Dv) {
#pragma unroll
  for (int ks = 0; ks < D / 16; ++ks) {
    const int d = ks * 16 + 2 * quad;
    const bool lo = d < Dv, hi = d + 8 < Dv;
    qa[ks][0] = (qp0 && lo) ? __ldg(reinterpret_cast<const unsigned int*>(qp0 + d)) : 0u;
    qa[ks][1] = (qp1 && lo) ? __ldg(reinterpret_cast<const unsigned int*>(qp1 + d)) : 0u;
    qa[ks][2] = (qp0 && hi) ? __ldg(reinterpret_cast<const unsigned int*>(qp0 + d + 8)) : 0u;
    qa[ks][3] = (qp1 && hi) ? __ldg(reinterpret_cast<const unsigned int*>(qp1 + d + 8)) : 0u;
  }
}

// S = Q K^T for the unit, scale into the log2 domain, causal mask (rows lim0 /
// lim1 attend positions <= lim), online-softmax update of (m, l, O), and
// O += P V.  tok_base = absolute position of the unit's first token; tokens at
// or past L are zeroed in V so stale non-finite cache contents cannot leak;
// the mask is evaluated only when the unit ends past `mask_from`.
template <typename T, int D>
__device__ __forceinline__ void attend_unit(uint32_t kbase, uint32_t vbase, const uint32_t (&qa)[D / 16][4],
                                            float (&o_acc)[D / 8][4], float& m0, float& m1, float& l0,
                                            float& l1, int tok_base, int L, int lim0, int lim1, int mask_from,
                                            float scale_log2, int lane) {
  constexpr int KSTEPS = D / 16;
  constexpr int NDT = D / 8;
  const int quad = lane & 3;

  float s_acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
  {
    const int tok = ((lane >> 4) << 3) | (lane & 7);
#pragma unroll
    for (int ks = 0; ks < KSTEPS; ++ks) {
      const int chunk = 2 * ks + ((lane >> 3) & 1);
      const uint32_t addr = kbase + (uint32_t)(chunk >> 3) * 2048u + (uint32_t)tok * 128u +
                            ((uint32_t)((chunk & 7) ^ (tok & 7)) << 4);
      uint32_t k0, k1, k2, k3;
      ldsm_x4(addr, k0, k1, k2, k3);
      Mma16816<T>::run(s_acc[0], qa[ks], k0, k1);
      Mma16816<T>::run(s_acc[1], qa[ks], k2, k3);
    }
  }

  float x[2][4];
#pragma unroll
  for (int n = 0; n < 2; ++n)
#pragma unroll
    for (int i = 0; i < 4; ++i) x[n][i] = s_acc[n][i] * scale_log2;
  if (tok_base + kUnitTokens - 1 > mask_from) {
#pragma unroll
    for (int n = 0; n < 2; ++n)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int tok = tok_base + n * 8 + 2 * quad + (i & 1);
        const int lim = (i < 2) ? lim0 : lim1;
        if (tok > lim) x[n][i] = -INFINITY;
      }
  }
  float mx0 = fmaxf(fmaxf(x[0][0], x[0][1]), fmaxf(x[1][0], x[1][1]));
  float mx1 = fmaxf(fmaxf(x[0][2], x[0][3]), fmaxf(x[1][2], x[1][3]));
  mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
  mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
  mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
  mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
  const float mn0 = fmaxf(m0, mx0);
  const float mn1 = fmaxf(m1, mx1);
  const float base0 = (mn0 == -INFINITY) ? 0.f : mn0;
  const float base1 = (mn1 == -INFINITY) ? 0.f : mn1;
  const float alpha0 = ex2(m0 - base0);
  const float alpha1 = ex2(m1 - base1);
  float pr[2][4];
#pragma unroll
  for (int n = 0; n < 2; ++n) {
    pr[n][0] = ex2(x[n][0] - base0);
    pr[n][1] = ex2(x[n][1] - base0);
    pr[n][2] = ex2(x[n][2] - base1);
    pr[n][3] = ex2(x[n][3] - base1);
  }
  l0 = l0 * alpha0 + (pr[0][0] + pr[0][1]) + (pr[1][0] + pr[1][1]);
  l1 = l1 * alpha1 + (pr[0][2] + pr[0][3]) + (pr[1][2] + pr[1][3]);
  m0 = mn0;
  m1 = mn1;
  // Once a row's running max settles, alpha is exactly 1: skip the rescale of
  // the accumulator unless some row of the warp moved its max in this unit.
  if (__any_sync(0xffffffffu, (alpha0 != 1.f) | (alpha1 != 1.f))) {
#pragma unroll
    for (int nd = 0; nd < NDT; ++nd) {
      o_acc[nd][0] *= alpha0;
      o_acc[nd][1] *= alpha0;
      o_acc[nd][2] *= alpha1;
      o_acc[nd][3] *= alpha1;
    }
  }
  uint32_t pa[4];
  pa[0] = pack2<T>(pr[0][0], pr[0][1]);
  pa[1] = pack2<T>(pr[0][2], pr[0][3]);
  pa[2] = pack2<T>(pr[1][0], pr[1][1]);
  pa[3] = pack2<T>(pr[1][2], pr[1][3]);
  // bf16 keeps 8 mantissa bits: P is also split into hi + lo (the residual,
  // rounded again) and both multiply V, so the P.V product carries ~16 bits of
  // P — as good as the reference's fp32 P for any softmax, including the
  // peaked ones of rows that attend only a few tokens.
  constexpr bool kSplitP = kSplitProbabilities<T>::value;
  uint32_t plo[4] = {0u, 0u, 0u, 0u};
  if (kSplitP) {
    plo[0] = pack2<T>(pr[0][0] - lo_half<T>(pa[0]), pr[0][1] - hi_half<T>(pa[0]));
    plo[1] = pack2<T>(pr[0][2] - lo_half<T>(pa[1]), pr[0][3] - hi_half<T>(pa[1]));
    plo[2] = pack2<T>(pr[1][0] - lo_half<T>(pa[2]), pr[1][1] - hi_half<T>(pa[2]));
    plo[3] = pack2<T>(pr[1][2] - lo_half<T>(pa[3]), pr[1][3] - hi_half<T>(pa[3]));
  }

  uint32_t vm0 = 0xffffffffu, vm1 = 0xffffffffu;
  if (tok_base + kUnitTokens > L) {
    const int t0 = tok_base + 2 * quad;
    vm0 = (t0 < L ? 0x0000ffffu : 0u) | (t0 + 1 < L ? 0xffff0000u : 0u);
    vm1 = (t0 + 8 < L ? 0x0000ffffu : 0u) | (t0 + 9 < L ? 0xffff0000u : 0u);
  }
  const int tok = (((lane >> 3) & 1) << 3) | (lane & 7);
#pragma unroll
  for (int nd = 0; nd < NDT; nd += 2) {
    const int chunk = nd + (lane >> 4);
    const uint32_t addr = vbase + (uint32_t)(chunk >> 3) * 2048u + (uint32_t)tok * 128u +
                          ((uint32_t)((chunk & 7) ^ (tok & 7)) << 4);
    uint32_t v0, v1, v2, v3;
    ldsm_x4_trans(addr, v0, v1, v2, v3);
    v0 &= vm0;
    v1 &= vm1;
    v2 &= vm0;
    v3 &= vm1;
    Mma16816<T>::run(o_acc[nd], pa, v0, v1);
    Mma16816<T>::run(o_acc[nd + 1], pa, v2, v3);
    if (kSplitP) {
      Mma16816<T>::run(o_acc[nd], plo, v0, v1);
      Mma16816<T>::run(o_acc[nd + 1], plo, v2, v3);
    }
  }
}

// Normalise and store the warp's rows (row pointers may be null for padding
// rows); columns at or past the head_dim Dv are not stored.
template <typename T, int D>
__device__ __forceinline__ void store_rows(T* op0, T* op1, const float (&o_acc)[D / 8][4], float l0, float l1,
                                           int quad, int Dv) {
  const float inv0 = l0 > 0.f ? 1.f / l0 : 0.f;
  const float inv1 = l1 > 0.f ? 1.f / l1 : 0.f;
#pragma unroll
  for (int nd = 0; nd < D / 8; ++nd) {
    const int d = nd * 8 + 2 * quad;
    if (d >= Dv) break;
    if (op0) *reinterpret_cast<uint32_t*>(op0 + d) = pack2<T>(o_acc[nd][0] * inv0, o_acc[nd][1] * inv0);
    if (op1) *reinterpret_cast<uint32_t*>(op1 + d) = pack2<T>(o_acc[nd][2] * inv1, o_acc[nd][3] * inv1);
  }
}

// store_rows for rows that also have a cascade prefix part: the prefix state
// of query rows ridx0 / ridx1 ((m, l) and the unnormalised accumulator, all
// splits already merged) is folded into the warp's running (m, l, acc) with a
// log-sum-exp merge, then normalised.  m0 / m1 are the rows' running maxima
// (log2 domain, -inf when nothing was attended), l0 / l1 their full sums;
// o_acc is consumed.
template <typename T, int D>
__device__ __forceinline__ void store_rows_folded(T* op0, T* op1, float (&o_acc)[D / 8][4], float m0, float m1,
                                                  float l0, float l1, long long ridx0, long long ridx1,
                                                  const DecodeParams& p, int quad) {
  const float2 ml0 = op0 ? __ldcg(&p.pre_ml[ridx0]) : make_float2(-INFINITY, 0.f);
  const float2 ml1 = op1 ? __ldcg(&p.pre_ml[ridx1]) : make_float2(-INFINITY, 0.f);
  const float M0 = fmaxf(m0, ml0.x), M1 = fmaxf(m1, ml1.x);
  const float base0 = (M0 == -INFINITY) ? 0.f : M0;
  const float base1 = (M1 == -INFINITY) ? 0.f : M1;
  const float w0 = ex2(m0 - base0), w1 = ex2(m1 - base1);      // this warp's part
  const float v0 = ex2(ml0.x - base0), v1 = ex2(ml1.x - base1);  // the prefix part
  l0 = fmaf(l0, w0, v0 * ml0.y);
  l1 = fmaf(l1, w1, v1 * ml1.y);
  const float* a0 = p.pre_acc + ridx0 * D + 2 * quad;
  const float* a1 = p.pre_acc + ridx1 * D + 2 * quad;
#pragma unroll
  for (int nd = 0; nd < D / 8; ++nd) {
    const float2 x0 = op0 ? __ldcg(reinterpret_cast<const float2*>(a0 + nd * 8)) : make_float2(0.f, 0.f);
    const float2 x1 = op1 ? __ldcg(reinterpret_cast<const float2*>(a1 + nd * 8)) : make_float2(0.f, 0.f);
    o_acc[nd][0] = fmaf(o_acc[nd][0], w0, v0 * x0.x);
    o_acc[nd][1] = fmaf(o_acc[nd][1], w0, v0 * x0.y);
    o_acc[nd][2] = fmaf(o_acc[nd][2], w1, v1 * x1.x);
    o_acc[nd][3] = fmaf(o_acc[nd][3], w1, v1 * x1.y);
  }
  store_rows<T, D>(op0, op1, o_acc, l0, l1, quad, p.Dv);
}

}  // namespace pa
