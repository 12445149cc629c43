// pa_capi.cu — the extern "C" boundary of the paged-decode library.
//
// Validates arguments (returning PA_ERR_* with a message, never aborting),
// encodes the TMA tensor maps of the two caches, sizes the grid from the
// device's SM count (never from device data, so calls are graph-capture safe)
// and launches the kernels on the caller's stream.  Nothing here allocates.
#include <cudaTypedefs.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <mutex>

#include "pa_common.cuh"
#include "pa_internal.h"

namespace {

thread_local char g_last_error[512] = "";
// Kernel launched by the last successful pa_decode on this host thread.
thread_local const char* g_last_kernel = "";

int fail(int status, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return status;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(PA_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

struct DeviceInfo {
  int num_sms = 0;
  int max_smem_optin = 0;
  bool prepared[3][2] = {{false, false}, {false, false}, {false, false}};  // [dtype][D==128]
  size_t prepared_smem[3][2] = {{0, 0}, {0, 0}, {0, 0}};
};

constexpr int kMaxDevices = 64;
DeviceInfo g_dev[kMaxDevices];
bool g_dev_valid[kMaxDevices] = {false};
std::mutex g_mu;

int device_info(int dev, DeviceInfo** out) {
  if (dev < 0 || dev >= kMaxDevices) return fail(PA_ERR_INVALID_ARGUMENT, "device %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_dev_valid[dev]) {
    cudaError_t e = cudaDeviceGetAttribute(&g_dev[dev].num_sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute(SM count)");
    e = cudaDeviceGetAttribute(&g_dev[dev].max_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute(smem opt-in)");
    g_dev_valid[dev] = true;
  }
  *out = &g_dev[dev];
  return PA_OK;
}

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

int get_encode(PFN_cuTensorMapEncodeTiled_v12000* fn) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_encode == nullptr) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || ptr == nullptr)
      return fail(PA_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
    g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  *fn = g_encode;
  return PA_OK;
}

// cuMemGetAddressRange (driver API), fetched like the tensor-map encoder: the
// allocation a pointer lies in, which is what CUDA IPC exports.
PFN_cuMemGetAddressRange_v3020 g_addr_range = nullptr;

int get_addr_range(PFN_cuMemGetAddressRange_v3020* fn) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_addr_range == nullptr) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuMemGetAddressRange", &ptr, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || ptr == nullptr)
      return fail(PA_ERR_CUDA, "cuMemGetAddressRange entry point unavailable");
    g_addr_range = reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(ptr);
  }
  *fn = g_addr_range;
  return PA_OK;
}

int allocation_base(const void* ptr, char** base) {
  PFN_cuMemGetAddressRange_v3020 fn = nullptr;
  int st = get_addr_range(&fn);
  if (st != PA_OK) return st;
  CUdeviceptr b = 0;
  size_t size = 0;
  CUresult r = fn(&b, &size, reinterpret_cast<CUdeviceptr>(ptr));
  if (r != CUDA_SUCCESS) return fail(PA_ERR_INVALID_ARGUMENT, "pointer is not device memory (CUresult %d)", (int)r);
  *base = reinterpret_cast<char*>(b);
  return PA_OK;
}

int elem_bytes(int dtype) { return dtype == PA_DTYPE_FLOAT32 ? 4 : 2; }

bool aligned_ptr(const void* p, int a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

constexpr size_t kAlign = 256;
size_t round_up(size_t x) { return (x + kAlign - 1) / kAlign * kAlign; }

int check_cache_view(const pa_cache_view& v, const char* name) {
  if (v.data == nullptr) return fail(PA_ERR_INVALID_ARGUMENT, "%s: null data pointer", name);
  if (v.num_blocks <= 0) return fail(PA_ERR_INVALID_ARGUMENT, "%s: num_blocks must be positive", name);
  if (v.stride_block <= 0 || v.stride_head <= 0 || v.stride_token <= 0)
    return fail(PA_ERR_INVALID_ARGUMENT, "%s: strides must be positive", name);
  return PA_OK;
}

// 4-D tensor map (head_dim, token, kv head, block) with 128-byte swizzle and a
// box of (64 elements, min(bs, 16) tokens, 1, 1).
int encode_cache_map(CUtensorMap* map, const pa_cache_view& v, int dtype, int D, int bs, int Hkv,
                     const char* name) {
  PFN_cuTensorMapEncodeTiled_v12000 enc;
  int st = get_encode(&enc);
  if (st != PA_OK) return st;
  const int e = elem_bytes(dtype);
  if (!aligned_ptr(v.data, 16))
    return fail(PA_ERR_UNSUPPORTED, "%s: base address must be 16-byte aligned", name);
  const int64_t sb[3] = {v.stride_token * e, v.stride_head * e, v.stride_block * e};
  for (int i = 0; i < 3; ++i)
    if (sb[i] % 16 != 0 || sb[i] >= (int64_t(1) << 40))
      return fail(PA_ERR_UNSUPPORTED, "%s: strides must be multiples of 16 bytes", name);
  cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)bs, (cuuint64_t)Hkv, (cuuint64_t)v.num_blocks};
  cuuint64_t strides[3] = {(cuuint64_t)sb[0], (cuuint64_t)sb[1], (cuuint64_t)sb[2]};
  cuuint32_t box[4] = {64u, (cuuint32_t)(bs < 16 ? bs : 16), 1u, 1u};
  cuuint32_t estr[4] = {1u, 1u, 1u, 1u};
  CUresult r = enc(map, dtype == PA_DTYPE_BFLOAT16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                   : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                   4, v.data, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(PA_ERR_UNSUPPORTED, "%s: cuTensorMapEncodeTiled failed (%d)", name, (int)r);
  return PA_OK;
}

// Kernel choice for multi-query tiles: PA_B200_MULTIQUERY=mma forces the
// mma.sync kernel (comparison / fallback); default is the tcgen05 kernel.
// PA_B200_MULTIQUERY: "mma" (the mma.sync kernel), "umma" (the one-SM tcgen05
// kernel), "umma2" (the SM-pair tcgen05 kernel where it applies); unset: auto.
constexpr int kPolicyAuto = 0, kPolicyMma = 1, kPolicyUmma = 2, kPolicyUmma2 = 3;
int multiquery_policy() {
  static int policy = -1;
  if (policy < 0) {
    const char* v = getenv("PA_B200_MULTIQUERY");
    policy = v == nullptr                ? kPolicyAuto
             : strcmp(v, "mma") == 0     ? kPolicyMma
             : strcmp(v, "umma") == 0    ? kPolicyUmma
             : strcmp(v, "umma2") == 0   ? kPolicyUmma2
                                         : kPolicyAuto;
  }
  return policy;
}

// The kernels' padded head width for a head_dim: the 16-bit tensor-core
// kernels tile 64 or 128 columns (TMA zero-fills the columns past the real
// head_dim), the fp32 kernel 32, 64 or 128.  0 when the head_dim is not served.
int padded_head_dim(int head_dim, int dtype) {
  if (head_dim <= 0) return 0;
  if (dtype == PA_DTYPE_FLOAT32) return head_dim <= 32 ? 32 : head_dim <= 64 ? 64 : head_dim <= 128 ? 128 : 0;
  if (head_dim % 8 != 0) return 0;  // rows of 16-byte pieces
  return head_dim <= 64 ? 64 : head_dim <= 128 ? 128 : 0;
}

struct DecodeShape {
  int G, GQ, NMG, slot_rows;
};

DecodeShape decode_shape(int Hq, int Hkv, int q_len) {
  DecodeShape s;
  s.G = Hq / Hkv;
  s.GQ = s.G * q_len;
  s.NMG = (s.GQ + 15) / 16;
  s.slot_rows = s.GQ < 16 ? s.GQ : 16;
  return s;
}

// Workspace: [status word | pad to 256][nw_total merge counters][2*nw_total partial
// slots].  The counters sit at a fixed offset whatever the call's shape, so a
// workspace shared by calls of different shapes keeps them at zero.
size_t workspace_bytes_impl(int slot_rows, int D, int nw_total) {
  return pa::kWsFixedBytes + pa::ws_counter_bytes(nw_total) + pa::ws_partial_bytes(nw_total, slot_rows, D);
}

// Fixed-point cumulative shares of the SMs from host weights; false (equal
// shares) when the weights do not describe this device or are not usable.
static_assert(sizeof(pa::SlotTiming) == sizeof(pa_sm_timing), "timing record layout");
static_assert(pa::kWsHeaderBytes == PA_WS_SM_TIMING_OFFSET, "timing record offset");
static_assert(pa::kMaxSlots == PA_MAX_SM_WEIGHTS, "SM weight count");
static_assert((pa::kMaxSlots + 1) * 4 <= (int)pa::kWsClaimBytes, "slot claim words");

bool slot_fractions(const float* w, int n, int num_sms, uint32_t* frac) {
  if (w == nullptr || n != num_sms || n <= 0 || n > pa::kMaxSlots) return false;
  double tot = 0.0;
  for (int i = 0; i < n; ++i) {
    if (!(w[i] > 0.f) || !(w[i] < 1e30f)) return false;
    tot += w[i];
  }
  const double one = (double)(1u << pa::kSlotFracBits);
  double run = 0.0;
  frac[0] = 0;
  for (int i = 0; i < n; ++i) {
    run += w[i];
    frac[i + 1] = i + 1 == n ? (1u << pa::kSlotFracBits) : (uint32_t)(run / tot * one + 0.5);
    if (frac[i + 1] <= frac[i]) return false;  // every share must be non-empty
  }
  return true;
}

// Cascade prefix pass: how many token ranges (splits) each group's prefix is
// cut into, and their length.  One split while the (group, kv head, 128-row
// tile) CTAs alone fill the GPU; otherwise enough ranges of >= 256 tokens to
// reach one CTA per SM, at most 16.
struct CascadeShape {
  int splits, split_tokens;
  size_t ml_bytes, acc_bytes, cnt_bytes;
};

CascadeShape cascade_shape(int num_sms, int num_groups, int max_members, int max_prefix, int Hkv, int GQ,
                           long long rows, int D) {
  CascadeShape c;
  // prefix-pass CTAs per split: kUmmaTileRows member rows each
  const long long tiles =
      (long long)num_groups * Hkv * (((long long)max_members * GQ + pa::kUmmaTileRows - 1) / pa::kUmmaTileRows);
  const int chunk = pa::kUmmaChunkTokens;
  const int prefix = max_prefix > 0 ? max_prefix : 0;
  int splits = 1;
  if (tiles > 0 && tiles < num_sms) {
    const long long want = (num_sms + tiles - 1) / tiles;
    const long long by_len = (prefix + 255) / 256;
    splits = (int)std::max(1LL, std::min({want, by_len, 16LL}));
  }
  int per = (prefix + splits - 1) / splits;
  per = std::max(chunk, (per + chunk - 1) / chunk * chunk);
  c.split_tokens = per;
  c.splits = std::max(1, (prefix + per - 1) / per);
  c.ml_bytes = round_up((size_t)c.splits * rows * 8);
  c.acc_bytes = round_up((size_t)c.splits * rows * D * 4);
  c.cnt_bytes = round_up((size_t)tiles * 4);
  return c;
}

}  // namespace

namespace pa {

int set_last_error(int status, const char* msg) { return fail(status, "%s", msg); }

size_t ws_counter_bytes(int nw_total) { return round_up((size_t)nw_total * 4); }

size_t ws_partial_bytes(int nw_total, int slot_rows, int D) {
  return round_up((size_t)2 * nw_total * slot_rows * (2 + D) * 4);
}

}  // namespace pa

extern "C" {

const char* pa_last_error(void) { return g_last_error; }

const char* pa_last_kernel(void) { return g_last_kernel; }

int32_t pa_version(void) { return 1 * 10000 + 0 * 100 + 0; }

size_t pa_decode_workspace_bytes(int32_t batch, int32_t num_q_heads, int32_t num_kv_heads,
                                 int32_t q_len, int32_t head_dim, int32_t dtype, int32_t device) {
  if (batch < 0 || num_q_heads <= 0 || num_kv_heads <= 0 || q_len <= 0 || head_dim <= 0 ||
      num_q_heads % num_kv_heads != 0)
    return 0;
  DeviceInfo* info = nullptr;
  if (device_info(device, &info) != PA_OK) return 0;
  const DecodeShape s = decode_shape(num_q_heads, num_kv_heads, q_len);
  if (dtype == PA_DTYPE_FLOAT32) return pa::kWsHeaderBytes;
  const int DP = padded_head_dim(head_dim, dtype);
  if (DP == 0) return pa::kWsHeaderBytes;  // not served: pa_decode itself reports it
  return workspace_bytes_impl(s.slot_rows, DP, info->num_sms * pa::kDecodeWarps);
}

int pa_workspace_init(void* workspace, size_t workspace_bytes, void* stream) {
  g_last_error[0] = 0;
  if (workspace == nullptr || workspace_bytes < pa::kWsHeaderBytes)
    return fail(PA_ERR_WORKSPACE, "workspace must be at least %zu bytes", pa::kWsHeaderBytes);
  cudaError_t e = cudaMemsetAsync(workspace, 0, workspace_bytes, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(workspace)");
  return PA_OK;
}

int pa_read_device_errors(void* device_word, uint32_t* host_flags, int32_t clear, void* stream) {
  g_last_error[0] = 0;
  if (device_word == nullptr || host_flags == nullptr)
    return fail(PA_ERR_INVALID_ARGUMENT, "null pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemcpyAsync(host_flags, device_word, sizeof(uint32_t), cudaMemcpyDeviceToHost, s);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyAsync(status word)");
  if (clear) {
    e = cudaMemsetAsync(device_word, 0, sizeof(uint32_t), s);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(status word)");
  }
  e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_fail(e, "cudaStreamSynchronize");
  return PA_OK;
}

int pa_kv_append(const pa_kv_append_args* a, void* stream) {
  g_last_error[0] = 0;
  if (a == nullptr) return fail(PA_ERR_INVALID_ARGUMENT, "null args");
  if (a->dtype < PA_DTYPE_FLOAT32 || a->dtype > PA_DTYPE_BFLOAT16)
    return fail(PA_ERR_UNSUPPORTED, "unsupported dtype %d", a->dtype);
  if (a->batch < 0 || a->q_len <= 0 || a->num_kv_heads <= 0 || a->head_dim <= 0 || a->block_size <= 0)
    return fail(PA_ERR_INVALID_ARGUMENT, "batch/q_len/num_kv_heads/head_dim/block_size must be positive");
  if (a->batch == 0) return PA_OK;
  if (a->key == nullptr || a->value == nullptr)
    return fail(PA_ERR_INVALID_ARGUMENT, "key and value must be given");
  int st = check_cache_view(a->key_cache, "key_cache");
  if (st != PA_OK) return st;
  st = check_cache_view(a->value_cache, "value_cache");
  if (st != PA_OK) return st;
  if (a->key_cache.num_blocks != a->value_cache.num_blocks)
    return fail(PA_ERR_INVALID_ARGUMENT, "key_cache and value_cache must have the same number of blocks");
  if (a->slot_mapping == nullptr) {
    if (a->block_tables == nullptr || a->positions == nullptr)
      return fail(PA_ERR_INVALID_ARGUMENT, "without slot_mapping, block_tables and positions are required");
    if (a->max_blocks <= 0) return fail(PA_ERR_INVALID_ARGUMENT, "max_blocks must be positive");
  }
  pa::AppendParams p;
  p.key = a->key;
  p.k_sb = a->key_stride_b;
  p.k_sh = a->key_stride_h;
  p.k_st = a->key_stride_t;
  p.value = a->value;
  p.v_sb = a->value_stride_b;
  p.v_sh = a->value_stride_h;
  p.v_st = a->value_stride_t;
  p.k_cache = a->key_cache.data;
  p.kc_sblk = a->key_cache.stride_block;
  p.kc_sh = a->key_cache.stride_head;
  p.kc_st = a->key_cache.stride_token;
  p.v_cache = a->value_cache.data;
  p.vc_sblk = a->value_cache.stride_block;
  p.vc_sh = a->value_cache.stride_head;
  p.vc_st = a->value_cache.stride_token;
  p.num_blocks = a->key_cache.num_blocks;
  p.slot_mapping = a->slot_mapping;
  p.block_tables = a->block_tables;
  p.bt_stride = a->block_table_stride;
  p.max_blocks = a->max_blocks;
  p.positions = a->positions;
  p.positions_is_int64 = a->positions_is_int64;
  p.position_offset = a->position_offset;
  p.B = a->batch;
  p.q_len = a->q_len;
  p.Hkv = a->num_kv_heads;
  p.D = a->head_dim;
  p.bs = a->block_size;
  p.elem_bytes = elem_bytes(a->dtype);
  p.error_flags = a->error_flags;
  cudaError_t e = pa::launch_kv_append(p, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "kv_append launch");
  return PA_OK;
}

size_t pa_cascade_workspace_bytes(int32_t batch, int32_t num_q_heads, int32_t num_kv_heads, int32_t q_len,
                                  int32_t head_dim, int32_t dtype, int32_t device, int32_t num_groups,
                                  int32_t max_members, int32_t max_prefix_len) {
  const size_t base = pa_decode_workspace_bytes(batch, num_q_heads, num_kv_heads, q_len, head_dim, dtype, device);
  if (base == 0 || dtype == PA_DTYPE_FLOAT32 || num_groups <= 0) return base;
  if (max_members <= 0 || max_prefix_len < 0) return 0;
  DeviceInfo* info = nullptr;
  if (device_info(device, &info) != PA_OK) return 0;
  const DecodeShape s = decode_shape(num_q_heads, num_kv_heads, q_len);
  const CascadeShape c = cascade_shape(info->num_sms, num_groups, max_members, max_prefix_len, num_kv_heads, s.GQ,
                                       (long long)batch * num_q_heads * q_len, padded_head_dim(head_dim, dtype));
  return base + c.ml_bytes + c.acc_bytes + c.cnt_bytes;
}

static int decode_impl(const pa_decode_args* a, const pa_prefix_groups* grp, const pa_gather_args* gat,
                       void* stream);

int pa_decode(const pa_decode_args* a, void* stream) { return decode_impl(a, nullptr, nullptr, stream); }

int pa_ipc_export(const void* device_ptr, pa_ipc_handle* handle) {
  g_last_error[0] = 0;
  if (device_ptr == nullptr || handle == nullptr) return fail(PA_ERR_INVALID_ARGUMENT, "null pointer");
  char* base = nullptr;
  int st = allocation_base(device_ptr, &base);
  if (st != PA_OK) return st;
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, base);
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcGetMemHandle");
  static_assert(sizeof(h) == PA_IPC_HANDLE_BYTES, "IPC handle size");
  memcpy(handle->bytes, &h, sizeof(h));
  handle->offset = static_cast<const char*>(device_ptr) - base;
  return PA_OK;
}

int pa_ipc_import(const pa_ipc_handle* handle, void** device_ptr) {
  g_last_error[0] = 0;
  if (handle == nullptr || device_ptr == nullptr) return fail(PA_ERR_INVALID_ARGUMENT, "null pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle->bytes, sizeof(h));
  void* base = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcOpenMemHandle");
  *device_ptr = static_cast<char*>(base) + handle->offset;
  return PA_OK;
}

int pa_ipc_release(void* device_ptr) {
  g_last_error[0] = 0;
  if (device_ptr == nullptr) return fail(PA_ERR_INVALID_ARGUMENT, "null pointer");
  char* base = nullptr;
  int st = allocation_base(device_ptr, &base);
  if (st != PA_OK) return st;
  cudaError_t e = cudaIpcCloseMemHandle(base);
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcCloseMemHandle");
  return PA_OK;
}

int pa_decode_gather(const pa_decode_args* a, const pa_gather_args* g, void* stream) {
  g_last_error[0] = 0;
  if (a == nullptr || g == nullptr) return fail(PA_ERR_INVALID_ARGUMENT, "null args");
  if (g->num_ranks < 1 || g->rank < 0 || g->rank >= g->num_ranks)
    return fail(PA_ERR_INVALID_ARGUMENT, "rank %d of %d ranks", g->rank, g->num_ranks);
  if (g->out_ranks == nullptr || g->flags_ranks == nullptr || g->epoch == nullptr || g->done_warps == nullptr)
    return fail(PA_ERR_INVALID_ARGUMENT, "gather needs out_ranks, flags_ranks, epoch and done_warps");
  if (g->head_offset < 0 || g->wait_ns <= 0)
    return fail(PA_ERR_INVALID_ARGUMENT, "head_offset must be >= 0 and wait_ns > 0");
  if (a->dtype == PA_DTYPE_FLOAT32) return fail(PA_ERR_UNSUPPORTED, "the fused gather supports fp16/bf16");
  return decode_impl(a, nullptr, g, stream);
}

int pa_decode_cascade(const pa_decode_args* a, const pa_prefix_groups* grp, void* stream) {
  g_last_error[0] = 0;
  if (grp == nullptr) return fail(PA_ERR_INVALID_ARGUMENT, "null prefix groups");
  if (grp->num_groups < 0) return fail(PA_ERR_INVALID_ARGUMENT, "num_groups must not be negative");
  if (grp->num_groups > 0) {
    if (grp->member_offsets == nullptr || grp->member_seqs == nullptr || grp->prefix_lens == nullptr ||
        grp->seq_group == nullptr)
      return fail(PA_ERR_INVALID_ARGUMENT, "prefix groups need member_offsets, member_seqs, prefix_lens, seq_group");
    if (grp->max_members <= 0 || grp->max_prefix_len < 0)
      return fail(PA_ERR_INVALID_ARGUMENT, "max_members must be positive and max_prefix_len non-negative");
  }
  return decode_impl(a, grp->num_groups > 0 ? grp : nullptr, nullptr, stream);
}

static int decode_impl(const pa_decode_args* a, const pa_prefix_groups* grp, const pa_gather_args* gat,
                       void* stream) {
  g_last_error[0] = 0;
  if (a == nullptr) return fail(PA_ERR_INVALID_ARGUMENT, "null args");
  const int dtype = a->dtype;
  if (dtype < PA_DTYPE_FLOAT32 || dtype > PA_DTYPE_BFLOAT16)
    return fail(PA_ERR_UNSUPPORTED, "unsupported dtype %d", dtype);
  if (a->batch < 0 || a->q_len <= 0 || a->num_q_heads <= 0 || a->num_kv_heads <= 0 ||
      a->head_dim <= 0 || a->block_size <= 0)
    return fail(PA_ERR_INVALID_ARGUMENT, "batch/q_len/heads/head_dim/block_size must be positive");
  if (a->num_q_heads % a->num_kv_heads != 0)
    return fail(PA_ERR_INVALID_ARGUMENT, "num_q_heads (%d) must be a multiple of num_kv_heads (%d)",
                a->num_q_heads, a->num_kv_heads);
  if (a->batch == 0) return PA_OK;
  if (a->query == nullptr || a->out == nullptr || a->block_tables == nullptr || a->context_lens == nullptr)
    return fail(PA_ERR_INVALID_ARGUMENT, "query, out, block_tables and context_lens must be given");
  if (a->max_blocks <= 0) return fail(PA_ERR_INVALID_ARGUMENT, "max_blocks must be positive");
  int st = check_cache_view(a->key_cache, "key_cache");
  if (st != PA_OK) return st;
  st = check_cache_view(a->value_cache, "value_cache");
  if (st != PA_OK) return st;
  if (a->key_cache.num_blocks != a->value_cache.num_blocks)
    return fail(PA_ERR_INVALID_ARGUMENT, "key_cache and value_cache must have the same number of blocks");
  const int Dv = a->head_dim, bs = a->block_size;
  const int D = padded_head_dim(Dv, dtype);  // the kernels' tile width
  if (D == 0)
    return fail(PA_ERR_UNSUPPORTED, "head_dim %d not served (%s)", Dv,
                dtype == PA_DTYPE_FLOAT32 ? "fp32: up to 128" : "fp16/bf16: a multiple of 8 up to 128");
  if ((int64_t)a->max_blocks * bs > (int64_t)1 << 30)
    return fail(PA_ERR_UNSUPPORTED, "max_blocks * block_size too large");
  if (!aligned_ptr(a->query, 4) || !aligned_ptr(a->out, 4) ||
      (dtype != PA_DTYPE_FLOAT32 && ((a->query_stride_b | a->query_stride_h | a->query_stride_t |
                                      a->out_stride_b | a->out_stride_h | a->out_stride_t) & 1) != 0))
    return fail(PA_ERR_UNSUPPORTED, "query/out rows must be 4-byte aligned");
  if (a->workspace == nullptr || a->workspace_bytes < pa::kWsHeaderBytes)
    return fail(PA_ERR_WORKSPACE, "a workspace of pa_decode_workspace_bytes() bytes is required");

  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  DeviceInfo* info = nullptr;
  st = device_info(dev, &info);
  if (st != PA_OK) return st;

  const DecodeShape s = decode_shape(a->num_q_heads, a->num_kv_heads, a->q_len);
  pa::DecodeParams p;
  memset(&p, 0, sizeof(p));
  p.q = a->query;
  p.q_sb = a->query_stride_b;
  p.q_sh = a->query_stride_h;
  p.q_st = a->query_stride_t;
  p.k_cache = a->key_cache.data;
  p.v_cache = a->value_cache.data;
  p.k_sblk = a->key_cache.stride_block;
  p.k_sh = a->key_cache.stride_head;
  p.k_st = a->key_cache.stride_token;
  p.v_sblk = a->value_cache.stride_block;
  p.v_sh = a->value_cache.stride_head;
  p.v_st = a->value_cache.stride_token;
  p.num_blocks = a->key_cache.num_blocks;
  p.block_tables = a->block_tables;
  p.bt_stride = a->block_table_stride;
  p.max_blocks = a->max_blocks;
  p.context_lens = a->context_lens;
  p.len_offset = a->len_offset;
  p.out = a->out;
  p.o_sb = a->out_stride_b;
  p.o_sh = a->out_stride_h;
  p.o_st = a->out_stride_t;
  p.B = a->batch;
  p.q_len = a->q_len;
  p.Hq = a->num_q_heads;
  p.Hkv = a->num_kv_heads;
  p.G = s.G;
  p.GQ = s.GQ;
  p.NMG = s.NMG;
  p.bs = bs;
  p.D = D;
  p.Dv = Dv;
  p.scale = a->scale;
  p.scale_log2 = a->scale * 1.4426950408889634f;
  p.status = static_cast<uint32_t*>(a->workspace);
  p.slot_rows = s.slot_rows;
  const bool pdl = a->allow_overlap_with_previous != 0;
  cudaStream_t strm = static_cast<cudaStream_t>(stream);

  if (dtype == PA_DTYPE_FLOAT32) {
    if (!aligned_ptr(a->key_cache.data, 4) || !aligned_ptr(a->value_cache.data, 4))
      return fail(PA_ERR_UNSUPPORTED, "cache base must be 4-byte aligned");
    g_last_kernel = "pa::decode_f32_kernel";
    e = pa::launch_decode_f32(p, pdl, strm);
    if (e != cudaSuccess) return cuda_fail(e, "decode_f32 launch");
    return PA_OK;
  }

  // fp16 / bf16: tensor-core kernel.
  if (bs < 8 || bs > 256 || (bs & (bs - 1)) != 0)
    return fail(PA_ERR_UNSUPPORTED, "fp16/bf16 decode needs a power-of-two block_size in [8, 256], got %d", bs);
  const int grid = info->num_sms;
  p.nw_total = grid * pa::kDecodeWarps;
  // tcgen05 kernels: each thread moves its query (and output) row in 16-byte pieces.
  const bool q_rows16 = aligned_ptr(a->query, 16) &&
                        ((a->query_stride_b | a->query_stride_h | a->query_stride_t) & 7) == 0;
  const bool rows16 = q_rows16 && aligned_ptr(a->out, 16) &&
                      ((a->out_stride_b | a->out_stride_h | a->out_stride_t) & 7) == 0;
  // Shared prefixes go through the tcgen05 prefix pass, which needs 16-byte
  // query rows; without them the plain decode computes the same result.
  const bool cascade = grp != nullptr && q_rows16;
  size_t need = workspace_bytes_impl(p.slot_rows, D, p.nw_total);
  CascadeShape cs = {1, pa::kUmmaChunkTokens, 0, 0, 0};
  if (cascade) {
    if ((long long)grp->max_members * s.GQ > (1LL << 30))
      return fail(PA_ERR_UNSUPPORTED, "max_members * rows per kv head too large");
    cs = cascade_shape(info->num_sms, grp->num_groups, grp->max_members, grp->max_prefix_len, p.Hkv, p.GQ,
                       (long long)p.B * p.Hq * p.q_len, D);
  }
  const size_t decode_need = need;
  need += cs.ml_bytes + cs.acc_bytes + cs.cnt_bytes;
  if (a->workspace_bytes < need)
    return fail(PA_ERR_WORKSPACE, "workspace too small: %zu bytes given, %zu needed", a->workspace_bytes, need);
  char* ws = static_cast<char*>(a->workspace);
  p.slot_timing = reinterpret_cast<pa::SlotTiming*>(ws + pa::kWsHeaderBytes);
  p.slot_claims = reinterpret_cast<int32_t*>(ws + pa::kWsHeaderBytes + pa::kWsTimingBytes);
  p.counters = reinterpret_cast<int32_t*>(ws + pa::kWsFixedBytes);
  p.partials = reinterpret_cast<float*>(ws + pa::kWsFixedBytes + pa::ws_counter_bytes(p.nw_total));
  if (slot_fractions(a->sm_weights, a->num_sm_weights, info->num_sms, p.slot_frac)) {
    p.n_slots = info->num_sms;
    p.timing_tag = a->sm_timing_tag;
  }
  if (gat != nullptr) {
    p.out_ranks = gat->out_ranks;
    p.flags_ranks = gat->flags_ranks;
    p.epoch = gat->epoch;
    p.done_warps = gat->done_warps;
    p.n_ranks = gat->num_ranks;
    p.rank = gat->rank;
    p.head_offset = gat->head_offset;
    p.wait_ns = gat->wait_ns;
  }
  if (cascade) {
    p.seq_group = grp->seq_group;
    p.group_prefix = grp->prefix_lens;
    p.member_off = grp->member_offsets;
    p.member_seq = grp->member_seqs;
    p.pre_ml = reinterpret_cast<float2*>(ws + decode_need);
    p.pre_acc = reinterpret_cast<float*>(ws + decode_need + cs.ml_bytes);
    p.pre_cnt = reinterpret_cast<int32_t*>(ws + decode_need + cs.ml_bytes + cs.acc_bytes);
    p.num_groups = grp->num_groups;
    p.max_members = grp->max_members;
    p.max_prefix = grp->max_prefix_len;
    p.splits = cs.splits;
    p.split_tokens = cs.split_tokens;
  }

  // Ring depth: as many 16-token stages per warp as shared memory allows (2..8).
  const size_t budget = (size_t)info->max_smem_optin - 128;  // static shared memory of the kernel (96 B)
  int stages = 8;
  while (stages >= 2 && pa::decode_mma_smem_bytes(D, p.B, stages, cascade) > budget) --stages;
  if (stages < 2)
    return fail(PA_ERR_UNSUPPORTED, "batch %d too large for the decode kernel's shared memory", p.B);
  p.stages = stages;
  const size_t smem = pa::decode_mma_smem_bytes(D, p.B, stages, cascade);

  CUtensorMap tmk, tmv;
  // the maps' rows are the real head_dim: TMA fills the columns past it with zeros
  st = encode_cache_map(&tmk, a->key_cache, dtype, Dv, bs, p.Hkv, "key_cache");
  if (st != PA_OK) return st;
  st = encode_cache_map(&tmv, a->value_cache, dtype, Dv, bs, p.Hkv, "value_cache");
  if (st != PA_OK) return st;

  {
    const int di = dtype, dj = D == 128 ? 1 : 0;
    std::lock_guard<std::mutex> lk(g_mu);
    if (!info->prepared[di][dj] || info->prepared_smem[di][dj] < smem) {
      e = pa::decode_mma_prepare(dtype, D, smem);
      if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(max dynamic smem)");
      info->prepared[di][dj] = true;
      info->prepared_smem[di][dj] = smem;
    }
  }
  // Many query rows per KV head (chunked prefill, long verify) with enough
  // 128-row tiles to fill the GPU: the multi-query kernel shares each K/V tile
  // across 128 rows.  Otherwise the split-K decode kernel.
  const long long prefill_tiles = (long long)p.B * p.Hkv * ((p.GQ + 127) / 128);
  if (gat != nullptr) {
    // the split-K decode kernel stores every output row to every rank and ends
    // with the ranks' flag exchange
    g_last_kernel = "pa::decode_mma_kernel<gather>";
    e = pa::launch_decode_mma(p, tmk, tmv, dtype, grid, smem, pdl, strm);
    if (e != cudaSuccess) return cuda_fail(e, "decode launch");
    return PA_OK;
  }
  if (cascade) {
    // Prefix pass (tcgen05), then the decode kernel over each member's own
    // tokens, which folds the prefix states in; it waits for the prefix grid.
    g_last_kernel = "pa::prefill_umma_kernel<prefix> + pa::decode_mma_kernel";
    bool prefix_pdl = pdl;
    if (cs.splits > 1) {
      // The split arrival counters sit after the shape-dependent regions, which
      // calls of other shapes reuse: start them at zero.
      e = cudaMemsetAsync(p.pre_cnt, 0, cs.cnt_bytes, strm);
      if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(prefix split counters)");
      prefix_pdl = false;  // the previous operation on the stream is now the memset
    }
    e = pa::launch_prefix_umma(p, tmk, tmv, dtype, prefix_pdl, strm);
    if (e != cudaSuccess) return cuda_fail(e, "cascade prefix launch");
    e = pa::launch_decode_mma(p, tmk, tmv, dtype, grid, smem, true, strm);
    if (e != cudaSuccess) return cuda_fail(e, "decode launch");
    return PA_OK;
  }
  if (p.GQ >= 64 && prefill_tiles >= info->num_sms) {
    const int pol = multiquery_policy();
    // SM pairs (cta_group::2): head_dim 128, blocks of 16 tokens or more.
    const bool pair_ok = rows16 && D == 128 && bs >= 16;
    if (pair_ok && pol == kPolicyUmma2) {
      g_last_kernel = "pa::prefill_umma2_kernel";
      e = pa::launch_prefill_umma2(p, tmk, tmv, dtype, pdl, strm);
      if (e != cudaSuccess) return cuda_fail(e, "tcgen05 SM-pair multi-query launch");
    } else if (rows16 && pol != kPolicyMma) {
      g_last_kernel = "pa::prefill_umma_kernel";
      e = pa::launch_prefill_umma(p, tmk, tmv, dtype, pdl, strm);
      if (e != cudaSuccess) return cuda_fail(e, "tcgen05 multi-query launch");
    } else {
      g_last_kernel = "pa::prefill_mma_kernel";
      e = pa::launch_prefill_mma(p, tmk, tmv, dtype, pdl, strm);
      if (e != cudaSuccess) return cuda_fail(e, "multi-query launch");
    }
    return PA_OK;
  }
  g_last_kernel = "pa::decode_mma_kernel";
  e = pa::launch_decode_mma(p, tmk, tmv, dtype, grid, smem, pdl, strm);
  if (e != cudaSuccess) return cuda_fail(e, "decode launch");
  return PA_OK;
}

}  // extern "C"
