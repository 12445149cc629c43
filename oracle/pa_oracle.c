/*
 * pa_oracle.c — CPU restatement of the reference's paged decode attention.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product links or calls this file;
 * only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use it,
 * as the checker.
 *
 * It restates, in plain C with fp32 arithmetic, the reference's per-row CPU
 * decode `_paged_attention_decode_torch`
 * (runtime/phase2/paged_attention_triton.py:663-704):
 *
 *   q = query[b, :, t, :].float()
 *   for each cache block of the row (block_size tokens, the last one partial):
 *       k, v   = cache[physical, kv_head, :take, :].float()
 *       scores = (q . k) * scaling                       (:694)
 *       m_new  = max(m, max(scores))                     (:695-696)
 *       p      = exp(scores - m_new); alpha = exp(m - m_new)  (:697-698)
 *       l      = l * alpha + sum(p)                      (:699)
 *       acc    = acc * alpha + p @ v                     (:700)
 *   out = acc / l                                        (:703, cast by the caller)
 *
 * extended to q_len > 1 with the causal limit of the reference's eager multi-
 * token path (runtime/phase2/block_paged_attention.py:50-59 with a causal
 * attention_mask): query token t attends positions 0 .. L - q_len + t, where
 * L = context_lens[b] + len_offset.  Probabilities stay in fp32 (the eager path
 * rounds them to the query dtype, which only adds noise).
 *
 * Inputs may be fp32, fp16 or bf16; they are widened to fp32 exactly.  The
 * output is fp32 [batch, num_q_heads, q_len, head_dim], contiguous.
 * Returns 0, or -1 when a block id is outside [0, num_blocks) or a row needs
 * more blocks than max_blocks (the reference raises IndexError there,
 * paged_kv_kernel.py:118-119, :263-264).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

enum { ORACLE_F32 = 0, ORACLE_F16 = 1, ORACLE_BF16 = 2 };

static float half_to_float(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  const uint32_t exp = (h >> 10) & 0x1fu;
  uint32_t mant = h & 0x3ffu;
  uint32_t bits;
  if (exp == 0) {
    if (mant == 0) {
      bits = sign;
    } else { /* subnormal: renormalise */
      int e = -1;
      do {
        ++e;
        mant <<= 1;
      } while ((mant & 0x400u) == 0);
      bits = sign | ((uint32_t)(127 - 15 - e) << 23) | ((mant & 0x3ffu) << 13);
    }
  } else if (exp == 31) {
    bits = sign | 0x7f800000u | (mant << 13);
  } else {
    bits = sign | ((exp + 127 - 15) << 23) | (mant << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

static float bf16_to_float(uint16_t h) {
  const uint32_t bits = (uint32_t)h << 16;
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

static float load(const void* base, int64_t idx, int dtype) {
  switch (dtype) {
    case ORACLE_F32:
      return ((const float*)base)[idx];
    case ORACLE_F16:
      return half_to_float(((const uint16_t*)base)[idx]);
    default:
      return bf16_to_float(((const uint16_t*)base)[idx]);
  }
}

int oracle_paged_decode(const void* query, int64_t q_sb, int64_t q_sh, int64_t q_st,
                        const void* key_cache, const void* value_cache, int64_t num_blocks,
                        int64_t c_sblk, int64_t c_sh, int64_t c_st, const int32_t* block_tables,
                        int64_t bt_stride, int32_t max_blocks, const int32_t* context_lens,
                        int32_t len_offset, float* out, int32_t batch, int32_t q_len,
                        int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                        int32_t block_size, int32_t dtype, float scaling, int32_t num_threads) {
  const int G = num_q_heads / num_kv_heads;
  const int D = head_dim;
  const int bs = block_size;
  int bad = 0;
  const int64_t rows = (int64_t)batch * num_q_heads * q_len;
#ifdef _OPENMP
  if (num_threads > 0) omp_set_num_threads(num_threads);
#pragma omp parallel for schedule(dynamic, 1) reduction(| : bad)
#endif
  for (int64_t row = 0; row < rows; ++row) {
    const int b = (int)(row / ((int64_t)num_q_heads * q_len));
    const int rem = (int)(row % ((int64_t)num_q_heads * q_len));
    const int hq = rem / q_len;
    const int t = rem % q_len;
    const int hk = hq / G; /* kv_indices = arange(num_heads) // num_kv_groups (:679) */
    float* o = out + row * D;
    float* q = (float*)malloc(sizeof(float) * D * 3 + sizeof(float) * bs);
    float* acc = q + D;
    float* scores = acc + D;
    for (int d = 0; d < D; ++d) q[d] = load(query, b * q_sb + hq * q_sh + t * q_st + d, dtype);
    for (int d = 0; d < D; ++d) acc[d] = 0.f;
    const int L = context_lens[b] + len_offset;
    int ntok = L - q_len + t + 1;
    if (ntok > L) ntok = L;
    if (ntok < 0) ntok = 0;
    float m = -INFINITY, l = 0.f;
    const int nblk = (ntok + bs - 1) / bs;
    if (nblk > max_blocks) bad |= 1;
    for (int blk = 0; blk < nblk && blk < max_blocks; ++blk) {
      const int32_t phys = block_tables[b * bt_stride + blk];
      if (phys < 0 || phys >= num_blocks) {
        bad |= 1;
        continue;
      }
      int take = ntok - blk * bs;
      if (take > bs) take = bs;
      const int64_t kb = (int64_t)phys * c_sblk + (int64_t)hk * c_sh;
      float bmax = -INFINITY;
      for (int j = 0; j < take; ++j) {
        float dot = 0.f;
        for (int d = 0; d < D; ++d) dot += q[d] * load(key_cache, kb + j * c_st + d, dtype);
        scores[j] = dot * scaling;
        if (scores[j] > bmax) bmax = scores[j];
      }
      const float m_new = m > bmax ? m : bmax;
      const float alpha = expf(m - m_new);
      float psum = 0.f;
      for (int j = 0; j < take; ++j) {
        scores[j] = expf(scores[j] - m_new);
        psum += scores[j];
      }
      l = l * alpha + psum;
      for (int d = 0; d < D; ++d) {
        float pv = 0.f;
        for (int j = 0; j < take; ++j) pv += scores[j] * load(value_cache, kb + j * c_st + d, dtype);
        acc[d] = acc[d] * alpha + pv;
      }
      m = m_new;
    }
    for (int d = 0; d < D; ++d) o[d] = l > 0.f ? acc[d] / l : 0.f;
    free(q);
  }
  return bad ? -1 : 0;
}
