// pa_internal.h — host-side plumbing shared by the kernel translation units and
// the C ABI (pa_capi.cu).  Not part of the public interface.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "../../include/paged_attention_b200.h"

namespace pa {

// Warps per CTA of the tensor-core decode kernel.  Each warp is a self-fed
// engine with its own ring of shared-memory stages.
constexpr int kDecodeWarps = 8;
// Multi-query (prefill) kernel: 8 consumer warps (128 query rows) + 1 producer.
constexpr int kPrefillWarps = 8;
constexpr int kPrefillThreads = (kPrefillWarps + 1) * 32;
constexpr int kPrefillStages = 6;
// tcgen05 multi-query kernel: 2 x 4 softmax warps (two 128-row tiles) + 1 TMA
// producer + 1 MMA-issue warp; the cascade's prefix pass adds a warp for its
// member table check (11 warps keep the 168-register budget that 10 have).
constexpr int umma_threads(bool prefix) { return (prefix ? 11 : 10) * 32; }
// Minimum number of 16-token units a warp's share of the flat work list holds
// before the kernel stops splitting the work further.
constexpr int kMinUnitsPerWarp = 8;
// Cost of a row's start and end in the decode kernel's stream-K split, in
// units: warps whose slices hold many short rows get fewer units.  Under the
// cascade a row end also folds the row's prefix state.
constexpr int kRowCostUnitsPlain = 1;
constexpr int kRowCostUnitsCascade = 4;
// Split rows of at most this many pieces are merged in the MMA fragment layout
// (all loads in flight at once); longer ones by the lane-parallel merge.
constexpr int kFragMergePieces = 4;
// Layout of the workspace: status word (header), per-SM timing records and
// slot claims, then merge counters, then partial slots.
constexpr size_t kWsHeaderBytes = 256;
// Per-SM shares of the decode kernel's cost line (large calls): at most this
// many SMs, fixed-point cumulative fractions with kSlotFracBits bits, used when
// every warp's share holds at least kWeightedMinUnitsPerWarp units of cost.
constexpr int kMaxSlots = 160;
constexpr int kSlotFracBits = 20;
constexpr int kWeightedMinUnitsPerWarp = 64;
// One timing record per slot (pa_sm_timing in the public header).
struct SlotTiming {
  unsigned long long t_start_ns, t_end_ns;
  uint32_t cost, smid, tag, pad;
};
constexpr size_t kWsTimingBytes = kMaxSlots * sizeof(SlotTiming);
constexpr size_t kWsClaimBytes = 1024;  // kMaxSlots claim words + the done counter, rounded
constexpr size_t kWsFixedBytes = kWsHeaderBytes + kWsTimingBytes + kWsClaimBytes;

// Kernel-side description of one decode call (passed by value).
struct DecodeParams {
  const void* q;
  int64_t q_sb, q_sh, q_st;
  const void* k_cache;  // used by the CUDA-core kernel (the tensor-core kernel uses TMA maps)
  const void* v_cache;
  int64_t k_sblk, k_sh, k_st;
  int64_t v_sblk, v_sh, v_st;
  int64_t num_blocks;
  const int32_t* block_tables;
  int64_t bt_stride;
  int32_t max_blocks;
  const int32_t* context_lens;
  int32_t len_offset;
  void* out;
  int64_t o_sb, o_sh, o_st;
  int32_t B, q_len, Hq, Hkv, G, GQ, NMG, bs, D;  // D: the kernels' padded head width (tile layout)
  int32_t Dv;        // the real head_dim (<= D): columns at or past it are masked
  float scale;       // softmax scale
  float scale_log2;  // scale * log2(e)
  uint32_t* status;  // device error word
  int32_t* counters; // [nw_total] merge arrival counters (kept at zero between calls)
  float* partials;   // [2 * nw_total] slots of (m, l, O) partial states
  int32_t slot_rows; // rows stored per partial slot
  int32_t nw_total;  // warps in the grid
  // Per-SM shares (n_slots > 0): slot s (taken by the CTA on SM s, or by any
  // CTA whose SM's slot is taken) covers the cost [C*f[s], C*f[s+1]) >> 20.
  int32_t n_slots;
  uint32_t slot_frac[kMaxSlots + 1];
  int32_t* slot_claims;      // [kMaxSlots] claim words, then the done counter (zero between calls)
  SlotTiming* slot_timing;   // [n_slots] records, written when timing_tag != 0
  uint32_t timing_tag;
  int32_t stages;    // shared-memory ring depth per warp
  // Shared prompt prefixes (pa_decode_cascade); seq_group is null otherwise.
  // The prefix kernel attends group g's member rows over tokens [0, P_g) with
  // P_g = prefix_lens[g] rounded down to whole 16-token units, in `splits`
  // ranges of split_tokens, and leaves per split and query row (b, hq, t)
  // (m, l) in pre_ml and the unnormalised accumulator in pre_acc, at row index
  // (b * Hq + hq) * q_len + t; the last split of a tile to finish merges all
  // splits into split 0.  The decode kernel starts each member at P_g and
  // folds that one state into its rows.
  const int32_t* seq_group;     // [B] group of each row, -1: none
  const int32_t* group_prefix;  // [num_groups] shared tokens
  const int32_t* member_off;    // [num_groups + 1]
  const int32_t* member_seq;    // member rows
  float2* pre_ml;               // [splits][B * Hq * q_len]; split 0 ends up holding the merged state
  float* pre_acc;               // [splits][B * Hq * q_len][D]
  int32_t* pre_cnt;             // [num_groups * Hkv * tiles] split arrival counters (zeroed per call)
  int32_t num_groups, max_members, max_prefix, splits, split_tokens;
  // Fused all-gather of KV-head-sharded decoding (pa_decode_gather); out_ranks
  // is null otherwise.  Output row (b, hq, t) goes to every rank's gathered
  // output at query head head_offset + hq; the grid's last warp then raises
  // this rank's flag (epoch) at every rank and waits for every rank's flag.
  void* const* out_ranks;       // [n_ranks] gathered outputs (this process's mappings)
  uint32_t* const* flags_ranks; // [n_ranks] flag arrays [n_ranks]
  uint32_t* epoch;              // this rank's call counter
  uint32_t* done_warps;         // warps finished in this call (zero between calls)
  int32_t n_ranks, rank, head_offset;
  int64_t wait_ns;
};

struct AppendParams {
  const void* key;
  int64_t k_sb, k_sh, k_st;
  const void* value;
  int64_t v_sb, v_sh, v_st;
  void* k_cache;
  int64_t kc_sblk, kc_sh, kc_st;
  void* v_cache;
  int64_t vc_sblk, vc_sh, vc_st;
  int64_t num_blocks;
  const int64_t* slot_mapping;
  const int32_t* block_tables;
  int64_t bt_stride;
  int32_t max_blocks;
  const void* positions;
  int32_t positions_is_int64;
  int32_t position_offset;
  int32_t B, q_len, Hkv, D, bs, elem_bytes;
  uint32_t* error_flags;
};

// Record the message pa_last_error() returns on this host thread; returns status.
int set_last_error(int status, const char* msg);

// Workspace layout helpers (bytes).
size_t ws_counter_bytes(int nw_total);
size_t ws_partial_bytes(int nw_total, int slot_rows, int D);

// Launchers (return cudaError_t of the launch).
cudaError_t launch_kv_append(const AppendParams& p, cudaStream_t stream);
// Mode follows the params: cascade when seq_group is set, fused gather when
// out_ranks is set, plain otherwise.
cudaError_t launch_decode_mma(const DecodeParams& p, const CUtensorMap& tmk, const CUtensorMap& tmv,
                              int dtype, int grid, size_t smem, bool pdl, cudaStream_t stream);
cudaError_t launch_decode_f32(const DecodeParams& p, bool pdl, cudaStream_t stream);
cudaError_t launch_prefill_mma(const DecodeParams& p, const CUtensorMap& tmk, const CUtensorMap& tmv, int dtype,
                               bool pdl, cudaStream_t stream);
cudaError_t launch_prefill_umma(const DecodeParams& p, const CUtensorMap& tmk, const CUtensorMap& tmv, int dtype,
                                bool pdl, cudaStream_t stream);
// The same on pairs of SMs (tcgen05 cta_group::2, clusters of 2 CTAs): head_dim
// 128 (p.D), block_size >= 16 only.
cudaError_t launch_prefill_umma2(const DecodeParams& p, const CUtensorMap& tmk, const CUtensorMap& tmv, int dtype,
                                 bool pdl, cudaStream_t stream);
// Prefix part of pa_decode_cascade (tcgen05): one CTA per (split, group, kv head,
// 128-row tile of the group's member rows).
cudaError_t launch_prefix_umma(const DecodeParams& p, const CUtensorMap& tmk, const CUtensorMap& tmv, int dtype,
                               bool pdl, cudaStream_t stream);
// Tokens per chunk of the tcgen05 kernels (prefix split ranges are multiples of it).
constexpr int kUmmaChunkTokens = 64;
// Query rows per CTA of the tcgen05 kernels (the prefix pass sizes its split
// counters by it).
constexpr int kUmmaTileRows = 256;

// Shared-memory bytes of the tensor-core kernel for given stage count.
size_t decode_mma_smem_bytes(int D, int B, int stages, bool cascade);
// Opt a kernel instantiation into large dynamic shared memory (once per device).
cudaError_t decode_mma_prepare(int dtype, int D, size_t smem);

}  // namespace pa
