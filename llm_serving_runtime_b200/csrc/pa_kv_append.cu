// pa_kv_append.cu — scatter a decode step's new K/V rows into the paged cache.
//
// Restates the scatter of GpuKVBlockPool.write_tokens_batch
// (runtime/phase2/paged_kv_kernel.py:217-227): token t of row b goes to
//   physical = block_tables[b, (start[b] + t) // bs],  offset = (start[b] + t) % bs,
//   cache[physical, h, offset, :] = new[b, h, t, :]
// or, in the slot_mapping form, to slot = physical * bs + offset given directly.
// The copy is bit-exact (raw bytes).  One thread moves one VEC-byte chunk; the
// grid covers (K|V) x token x kv head x chunk, so a row of 256 bytes is moved
// by 16 threads with 16-byte loads/stores — fully coalesced on both sides.
#include "pa_common.cuh"
#include "pa_internal.h"

namespace pa {

template <int VEC>
struct VecType;
template <>
struct VecType<16> {
  using type = uint4;
};
template <>
struct VecType<8> {
  using type = uint2;
};
template <>
struct VecType<4> {
  using type = uint32_t;
};
template <>
struct VecType<2> {
  using type = uint16_t;
};

template <int VEC>
__global__ void __launch_bounds__(256) kv_append_kernel(const AppendParams p) {
  using V = typename VecType<VEC>::type;
  // The decode kernel that follows may start its prologue right away; its
  // griddepcontrol.wait still waits for every write below.
  pdl_launch_dependents();

  const int chunks = (p.D * p.elem_bytes) / VEC;
  const long long per_tensor = (long long)p.B * p.q_len * p.Hkv * chunks;
  const long long total = 2 * per_tensor;
  const long long step = (long long)gridDim.x * blockDim.x;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += step) {
    const int which = i >= per_tensor;  // 0: key, 1: value
    long long j = which ? i - per_tensor : i;
    const int c = (int)(j % chunks);
    j /= chunks;
    const int h = (int)(j % p.Hkv);
    const int token = (int)(j / p.Hkv);  // b * q_len + t
    const int b = token / p.q_len;
    const int t = token - b * p.q_len;
    // Only one thread per (token, head) reports an error, to keep atomics rare.
    const bool reporter = (which == 0) && (c == 0);

    long long blk, off;
    if (p.slot_mapping != nullptr) {
      const long long slot = p.slot_mapping[token];
      if (slot < 0) continue;  // padding token
      blk = slot / p.bs;
      off = slot - blk * p.bs;
    } else {
      const long long start = p.positions_is_int64
                                  ? static_cast<const int64_t*>(p.positions)[b]
                                  : (long long)static_cast<const int32_t*>(p.positions)[b];
      const long long pos = start + p.position_offset + t;
      if (pos < 0) {
        if (reporter) raise_flag(p.error_flags, PA_DEVERR_SLOT_RANGE);
        continue;
      }
      const long long lb = pos / p.bs;
      if (lb >= p.max_blocks) {  // paged_kv_kernel.py:221-222 "block table underrun"
        if (reporter) raise_flag(p.error_flags, PA_DEVERR_TABLE_UNDERRUN);
        continue;
      }
      blk = p.block_tables[(long long)b * p.bt_stride + lb];
      off = pos - lb * p.bs;
      if (blk < 0) {
        if (reporter) raise_flag(p.error_flags, PA_DEVERR_BLOCK_ID_RANGE);
        continue;
      }
    }
    if (blk >= p.num_blocks) {
      if (reporter)
        raise_flag(p.error_flags,
                   p.slot_mapping != nullptr ? PA_DEVERR_SLOT_RANGE : PA_DEVERR_BLOCK_ID_RANGE);
      continue;
    }

    const char* src;
    char* dst;
    if (which == 0) {
      src = static_cast<const char*>(p.key) +
            ((long long)b * p.k_sb + (long long)h * p.k_sh + (long long)t * p.k_st) * p.elem_bytes;
      dst = static_cast<char*>(p.k_cache) +
            (blk * p.kc_sblk + (long long)h * p.kc_sh + off * p.kc_st) * p.elem_bytes;
    } else {
      src = static_cast<const char*>(p.value) +
            ((long long)b * p.v_sb + (long long)h * p.v_sh + (long long)t * p.v_st) * p.elem_bytes;
      dst = static_cast<char*>(p.v_cache) +
            (blk * p.vc_sblk + (long long)h * p.vc_sh + off * p.vc_st) * p.elem_bytes;
    }
    *reinterpret_cast<V*>(dst + (long long)c * VEC) =
        *reinterpret_cast<const V*>(src + (long long)c * VEC);
  }
}

cudaError_t launch_kv_append(const AppendParams& p, cudaStream_t stream) {
  const int row_bytes = p.D * p.elem_bytes;
  // Largest vector width that divides the row and every base/stride in bytes.
  auto aligned = [&](int vec) {
    auto ok_ptr = [&](const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) % vec) == 0; };
    auto ok_str = [&](int64_t s) { return ((s * p.elem_bytes) % vec) == 0; };
    return row_bytes % vec == 0 && ok_ptr(p.key) && ok_ptr(p.value) && ok_ptr(p.k_cache) &&
           ok_ptr(p.v_cache) && ok_str(p.k_sb) && ok_str(p.k_sh) && ok_str(p.k_st) &&
           ok_str(p.v_sb) && ok_str(p.v_sh) && ok_str(p.v_st) && ok_str(p.kc_sblk) &&
           ok_str(p.kc_sh) && ok_str(p.kc_st) && ok_str(p.vc_sblk) && ok_str(p.vc_sh) &&
           ok_str(p.vc_st);
  };
  int vec = 2;
  if (aligned(16))
    vec = 16;
  else if (aligned(8))
    vec = 8;
  else if (aligned(4))
    vec = 4;
  const long long total = 2LL * p.B * p.q_len * p.Hkv * (row_bytes / vec);
  if (total == 0) return cudaSuccess;
  const int threads = 256;
  long long blocks = (total + threads - 1) / threads;
  if (blocks > 148LL * 16) blocks = 148LL * 16;
  switch (vec) {
    case 16:
      kv_append_kernel<16><<<(unsigned)blocks, threads, 0, stream>>>(p);
      break;
    case 8:
      kv_append_kernel<8><<<(unsigned)blocks, threads, 0, stream>>>(p);
      break;
    case 4:
      kv_append_kernel<4><<<(unsigned)blocks, threads, 0, stream>>>(p);
      break;
    default:
      kv_append_kernel<2><<<(unsigned)blocks, threads, 0, stream>>>(p);
      break;
  }
  return cudaGetLastError();
}

}  // namespace pa
