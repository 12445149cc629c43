// pa_decode_mma.cu — paged decode attention for fp16 / bf16 on sm_100a.
//
// What it computes (per sequence b, KV head h, query row (g, t)):
//   out[b, h*G+g, t, :] = softmax_j( q . k_j * scale ) @ v_j   over cached tokens
//   j = 0 .. L_b - q_len + t  (causal over the q_len new tokens; q_len = 1: all L_b)
// which is the math of the reference's decode kernels and CPU path
// (runtime/phase2/paged_attention_triton.py:148-243 and :663-704): fp32 scores,
// online softmax with running max m, sum l and accumulator acc, out = acc / l.
//
// How (B200-first):
//  * Work is one flat list of 16-token "units" ordered (sequence, kv head,
//    query-row group, unit).  Every warp of the persistent grid takes a
//    contiguous slice of it of equal cost (stream-K), a row costing its units
//    plus a fixed few for its start and end, so ragged / log-uniform lengths
//    and many short rows balance alike.  A slice that covers a whole (sequence, head) writes
//    the output directly; a row cut by a slice boundary leaves (m, l, acc)
//    partials in the workspace, and the last warp to finish that row merges
//    them with a log-sum-exp reduction (arrival counter, reset after use; one
//    counter per warp of the grid, so the workspace layout is shape-independent).
//  * GQA packing: the G query heads (times q_len query tokens) that read one KV
//    head form the 16 rows of an m16n8k16 tile, so each K/V tile is read from
//    HBM once for the whole group.
//  * Each warp is a self-fed engine: its lane 0 issues 4-D TMA tile loads
//    (128-byte swizzle, each CTA loading only for itself) of the unit's K and V tiles into a ring of
//    `stages` shared-memory slots tracked by mbarriers; the warp keeps `stages`
//    units in flight while it computes the oldest one.  Block-table entries are
//    fetched 32 at a time with one coalesced load and shuffled to lane 0.
//  * QK^T and PV run on tensor cores (ldmatrix + mma.sync m16n8k16, fp32
//    accumulate); the online softmax uses quad shuffles and ex2.
#include <math.h>

#include "pa_common.cuh"
#include "pa_internal.h"
#include "pa_tile_math.cuh"

namespace pa {

namespace {

struct Cursor {
  int b;   // sequence
  int h;   // kv head
  int mg;  // query-row group (16 rows of the G * q_len rows of this kv head)
  int u;   // unit within the row
  int n;   // units in the row
};

}  // namespace

// Query rows of one kv head are ordered token-major: row qr is query token
// qr / G of query head h*G + qr % G, so a 16-row group holds consecutive tokens
// of every head that reads this kv head.  A group whose latest token is t_max
// attends positions 0 .. L - q_len + t_max: it scans that many 16-token units.
__device__ __forceinline__ int group_units(int L, int mg, const DecodeParams& p) {
  const int last_row = min(16 * mg + 15, p.GQ - 1);
  const int lim = L - p.q_len + last_row / p.G;  // last attendable position
  return lim < 0 ? 0 : (lim + kUnitTokens) / kUnitTokens;
}

// The fused all-gather's end of a call, run by the grid's last warp: raise
// this rank's flag (the call's epoch) at every rank with a system-scope release
// and wait, at most p.wait_ns, until every rank's flag in this rank's array
// reached the epoch.  The other ranks' output rows in this rank's gathered
// output are visible once their flags are (each warp fenced its stores before
// counting itself done).  A peer's flag may already be one call ahead (it
// finished the next call, whose rows go to the other gathered buffer); more
// than one is impossible while the ranks make the same calls.
//
// Once a wait runs out, or a peer's flag is out of step, the ranks no longer
// agree on which call is which, and a later call could take a peer's rows of a
// different call without noticing.  So the rank poisons the gather: bit 31 of
// its epoch and of its flag at every rank.  Every later call of this rank, and
// of every peer that reads the flag, then reports PA_DEVERR_GATHER at once,
// without waiting, until the ranks set up fresh flags together.
constexpr uint32_t kGatherPoison = 0x80000000u;

__device__ __noinline__ void gather_barrier(uint32_t* const* flags_ranks, uint32_t* epoch, uint32_t* done_warps,
                                            int n_ranks, int rank, int64_t wait_ns, uint32_t* status, int lane) {
  __threadfence();
  const uint32_t cur = *epoch;
  __syncwarp();
  if (cur & kGatherPoison) {
    if (lane == 0) *done_warps = 0u;
    for (int i = lane; i < n_ranks; i += 32) st_release_sys(flags_ranks[i] + rank, cur);
    if (lane == 0) raise_flag(status, PA_DEVERR_GATHER);
    return;
  }
  const uint32_t e = (cur + 1u) & ~kGatherPoison;
  if (lane == 0) {
    *done_warps = 0u;  // ready for the next call
    *epoch = e;
  }
  __threadfence_system();
  for (int i = lane; i < n_ranks; i += 32) st_release_sys(flags_ranks[i] + rank, e);
  const uint32_t* mine = flags_ranks[rank];
  bool timed_out = false, out_of_step = false;
  for (int i = lane; i < n_ranks; i += 32) {
    const uint64_t t0 = global_ns();
    for (;;) {
      const uint32_t f = ld_acquire_sys(mine + i);
      const uint32_t d = (f - e) & ~kGatherPoison;
      if (f & kGatherPoison) {
        out_of_step = true;
        break;
      }
      if (d <= 1u) break;  // this call, or the peer is one call ahead
      if (d < (kGatherPoison >> 1)) {  // ahead by more than one call
        out_of_step = true;
        break;
      }
      if (global_ns() - t0 > (uint64_t)wait_ns) {
        timed_out = true;
        break;
      }
      __nanosleep(256);
    }
  }
  const bool any_timeout = __any_sync(0xffffffffu, timed_out);
  if (__any_sync(0xffffffffu, timed_out || out_of_step)) {
    const uint32_t poisoned = e | kGatherPoison;
    if (lane == 0) *epoch = poisoned;
    __threadfence_system();
    for (int i = lane; i < n_ranks; i += 32) st_release_sys(flags_ranks[i] + rank, poisoned);
    if (lane == 0) raise_flag(status, PA_DEVERR_GATHER | (any_timeout ? PA_DEVERR_WAIT_TIMEOUT : 0u));
  }
}

// kMode 1 (cascade): the call carries shared-prefix groups (pa_decode_cascade);
// each member's prefix units are skipped and the prefix states folded into its
// rows.  kMode 2 (gather): output rows go to every rank's gathered output
// (pa_decode_gather).  kMode 0: plain decode.
template <typename T, int D, int kMode>
__global__ void __launch_bounds__(kDecodeWarps * 32, 1)
    decode_mma_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
                      const DecodeParams p) {
  constexpr int KSTEPS = D / 16;             // k-steps of QK^T
  constexpr int NDT = D / 8;                 // n-tiles of PV
  constexpr int HALVES = D / 64;             // 128-byte column halves of a tile row
  constexpr uint32_t TILE_BYTES = 16 * D * 2;  // one 16-token K (or V) tile
  constexpr uint32_t STAGE_BYTES = 2 * TILE_BYTES;
  constexpr int DPL = D / 32;                // dims per lane in the merge

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_addr(smem_raw);
  const uint32_t pad = (1024u - (raw_addr & 1023u)) & 1023u;
  uint8_t* smem = smem_raw + pad;
  const int stages = p.stages;
  const uint32_t ring_addr = smem_addr(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + (size_t)kDecodeWarps * stages * STAGE_BYTES);
  int* s_lens = reinterpret_cast<int*>(bars + kDecodeWarps * stages);
  int* s_pref = s_lens + p.B;
  int* s_rpref = s_pref + p.B + 1;  // exclusive prefix of rows with units, per sequence
  // Cascade (shared prefixes): the prefix kernel has attended each member's
  // first s_u0[b] units; the work list starts every sequence after them.
  int* s_u0 = s_rpref + p.B + 1;
  constexpr bool cascade = kMode == 1;
  constexpr bool gather = kMode == 2;
  __shared__ int s_warp_tot[kDecodeWarps];
  __shared__ int s_warp_rows[kDecodeWarps];

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int B = p.B;

  if (lane == 0) {
    for (int s = 0; s < stages; ++s) mbar_init(smem_addr(&bars[warp * stages + s]), 1);
  }
  if (tid == 0) {
    prefetch_tensormap(&tmk);
    prefetch_tensormap(&tmv);
  }

  // ---- prologue: attended lengths and the exclusive prefix of units per sequence.
  // (context_lens and block tables are not written by the append kernel, so
  // this runs before griddepcontrol.wait and overlaps it.)
  {
    const int cap = p.max_blocks * p.bs;
    const int nthr = (int)blockDim.x;
    const int per = (B + nthr - 1) / nthr;
    const int beg = min(B, tid * per);
    const int end = min(B, beg + per);
    int local = 0, local_rows = 0;
    for (int b = beg; b < end; ++b) {
      int L = p.context_lens[b] + p.len_offset;
      if (L > cap) {
        if (blockIdx.x == 0) raise_flag(p.status, PA_DEVERR_TABLE_UNDERRUN);
        L = cap;
      }
      if (L < 0) L = 0;
      s_lens[b] = L;
      int u0 = 0;
      if (cascade) {
        const int gi = p.seq_group[b];
        if (gi >= 0 && gi < p.num_groups) u0 = cascade_prefix_tokens(p, gi) / kUnitTokens;
        s_u0[b] = u0;
      }
      int units = 0, rows = 0;
      for (int mg = 0; mg < p.NMG; ++mg) {
        const int n = max(0, group_units(L, mg, p) - u0);
        units += n;
        rows += n > 0;
      }
      local += units * p.Hkv;
      local_rows += rows * p.Hkv;
    }
    int incl = local, incl_r = local_rows;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      const int vr = __shfl_up_sync(0xffffffffu, incl_r, o);
      if (lane >= o) {
        incl += v;
        incl_r += vr;
      }
    }
    if (lane == 31) {
      s_warp_tot[warp] = incl;
      s_warp_rows[warp] = incl_r;
    }
    __syncthreads();
    int run = incl - local, run_r = incl_r - local_rows;
    for (int w = 0; w < warp; ++w) {
      run += s_warp_tot[w];
      run_r += s_warp_rows[w];
    }
    for (int b = beg; b < end; ++b) {
      s_pref[b] = run;
      s_rpref[b] = run_r;
      int units = 0, rows = 0;
      for (int mg = 0; mg < p.NMG; ++mg) {
        const int n = max(0, group_units(s_lens[b], mg, p) - (cascade ? s_u0[b] : 0));
        units += n;
        rows += n > 0;
      }
      run += units * p.Hkv;
      run_r += rows * p.Hkv;
    }
    if (tid == nthr - 1) {
      s_pref[B] = run;
      s_rpref[B] = run_r;
    }
  }
  fence_mbar_init();
  __syncthreads();

  // Output row (b, query head hq, token t) in destination dst: this call's
  // output, or under the fused gather rank dst's gathered output.
  const int n_dst = gather ? p.n_ranks : 1;
  auto out_row = [&](int dst, int b, int hq, int t) -> T* {
    T* base = gather ? static_cast<T*>(p.out_ranks[dst]) : static_cast<T*>(p.out);
    return base + (long long)b * p.o_sb + (long long)((gather ? p.head_offset : 0) + hq) * p.o_sh +
           (long long)t * p.o_st;
  };
  // Every warp passes here exactly once, when it has stored all its rows.
  auto finish_warp = [&]() {
    if constexpr (gather) {
      __threadfence_system();  // this warp's row stores, local and remote, before its count
      __syncwarp();
      int last = 0;
      if (lane == 0) last = atomicAdd(p.done_warps, 1u) == gridDim.x * kDecodeWarps - 1u;
      if (__shfl_sync(0xffffffffu, last, 0))
        gather_barrier(p.flags_ranks, p.epoch, p.done_warps, p.n_ranks, p.rank, p.wait_ns, p.status, lane);
    }
  };

  // Units of row group mg of sequence b in the work list.
  auto units_of = [&](int b, int mg) -> int {
    const int n = group_units(s_lens[b], mg, p);
    return cascade ? max(0, n - s_u0[b]) : n;
  };

  // Row groups with nothing to attend get no unit: their rows are zero, or,
  // under the cascade, the normalised prefix part alone.
  auto fill_empty_rows = [&]() {
    for (int b = blockIdx.x; b < B; b += gridDim.x) {
      const bool pre = cascade && s_u0[b] > 0;
      for (int mg = 0; mg < p.NMG; ++mg) {
        if (units_of(b, mg) != 0) continue;
        const int rows = min(16, p.GQ - 16 * mg);
        for (int i = tid; i < p.Hkv * rows * (D / 2); i += blockDim.x) {
          const int d2 = i % (D / 2);
          const int hr = i / (D / 2);
          const int h = hr / rows;
          const int qr = 16 * mg + (hr - h * rows);
          const int t = qr / p.G, g = qr - (qr / p.G) * p.G;
          uint32_t v = 0u;
          if (pre) {  // merged prefix state: out = acc / l
            const long long ridx = ((long long)b * p.Hq + h * p.G + g) * p.q_len + t;
            const float lsum = __ldcg(&p.pre_ml[ridx]).y;
            const float2 a = __ldcg(reinterpret_cast<const float2*>(p.pre_acc + ridx * D + 2 * d2));
            const float inv = lsum > 0.f ? 1.f / lsum : 0.f;
            v = pack2<T>(a.x * inv, a.y * inv);
          }
          if (2 * d2 < p.Dv)
            for (int dst = 0; dst < n_dst; ++dst)
              *reinterpret_cast<uint32_t*>(out_row(dst, b, h * p.G + g, t) + 2 * d2) = v;
        }
      }
    }
  };
  if constexpr (!cascade) fill_empty_rows();

  // Up to the first K/V load, the slices below read only the lengths and the
  // block tables, which the previous kernel (the append, or under the cascade
  // the prefix pass) does not write: they are worked out, and each warp's
  // first block-table window loaded, before waiting for that kernel.
  const long long W = s_pref[B];
  // Slices are equal in cost, not in units: a row (a row group of one
  // sequence and kv head with units) costs its units plus kRowCostUnits for
  // what a row start and end take (query load, output store, fold, merge).
  // Unit u of a row whose cost starts at rc sits at cost position
  // rc + kRowCostUnits + u; a warp's slice is the units whose positions fall
  // in its equal share of the total cost C.
  constexpr int kRowCostUnits = cascade ? kRowCostUnitsCascade : kRowCostUnitsPlain;
  const long long C = W + (long long)kRowCostUnits * s_rpref[B];
  long long nw_eff = (C + kMinUnitsPerWarp - 1) / kMinUnitsPerWarp;
  if (nw_eff > p.nw_total) nw_eff = p.nw_total;
  if (nw_eff < 1) nw_eff = 1;
  // Per-SM shares.  SMs stream at different speeds (up to ~10 % apart, in a
  // pattern fixed by where they sit), so with equal shares the call ends with
  // the slowest SMs.  Large calls given per-SM weights (p.n_slots, one slot per
  // SM) instead cut the cost line into one share per slot in proportion to
  // its SM's measured speed, and each CTA takes the slot of the SM it runs on
  // (or, should that one be taken, the first free one: the grid has one CTA
  // per slot, so every slot is taken exactly once).  The 8 warps of a slot
  // split it equally.  Which CTA runs a slot does not change the numbers:
  // shares, pieces and merges follow the slots.
  const bool weighted = p.n_slots > 0 && p.n_slots == (int)gridDim.x &&
                        nw_eff == (long long)p.n_slots * kDecodeWarps &&
                        C >= nw_eff * (long long)kWeightedMinUnitsPerWarp;
  __shared__ int s_slot;
  __shared__ unsigned long long s_t0, s_t1;
  __shared__ int s_warps_out;
  if (weighted) {
    if (tid == 0) {
      const int smid = (int)smid_u32();
      int sl = -1;
      if (smid < p.n_slots && atomicCAS(&p.slot_claims[smid], 0, 1) == 0) sl = smid;
      for (int i = 0; sl < 0 && i < p.n_slots; ++i)
        if (atomicCAS(&p.slot_claims[i], 0, 1) == 0) sl = i;
      s_slot = sl;
      s_t0 = ~0ull;
      s_t1 = 0ull;
      s_warps_out = 0;
    }
    __syncthreads();
  }
  const int gw = weighted ? s_slot * kDecodeWarps + warp : blockIdx.x * kDecodeWarps + warp;
  // Cost at which slot s starts (s = n_slots: C).
  auto slot_bound = [&](int sl) -> long long { return (C * (long long)p.slot_frac[sl]) >> kSlotFracBits; };
  // Cost at which global warp g's share starts (g = nw_eff: C).
  auto warp_start = [&](int g) -> long long {
    if (!weighted) return C * g / nw_eff;
    const int sl = g / kDecodeWarps, w = g - sl * kDecodeWarps;
    const long long b0 = slot_bound(sl);
    return w == 0 ? b0 : b0 + (slot_bound(sl + 1) - b0) * w / kDecodeWarps;
  };
  // The global warp whose share holds cost position x (0 <= x < C).
  auto warp_at_cost = [&](long long x) -> int {
    if (!weighted) return (int)(((x + 1) * nw_eff - 1) / C);
    int lo = 0, hi = p.n_slots - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (slot_bound(mid) <= x)
        lo = mid;
      else
        hi = mid - 1;
    }
    const long long b0 = slot_bound(lo), len = slot_bound(lo + 1) - b0;
    return lo * kDecodeWarps + (int)(((x - b0 + 1) * kDecodeWarps - 1) / len);
  };
  // Every warp of a weighted call counts itself out once: the CTA's last one
  // writes the slot's timing record (when asked), and the grid's last one
  // clears the slot claims for the next call.
  auto leave_weighted = [&]() {
    if (!weighted) return;
    __syncwarp();
    if (lane == 0) {
      const unsigned long long t = (unsigned long long)global_ns();
      atomicMax(&s_t1, t);
      __threadfence_block();
      if (atomicAdd(&s_warps_out, 1) == kDecodeWarps - 1 && p.timing_tag != 0u && s_slot >= 0) {
        __threadfence_block();
        SlotTiming* r = p.slot_timing + s_slot;
        r->t_start_ns = s_t0;
        r->t_end_ns = s_t1;
        r->cost = (uint32_t)(slot_bound(s_slot + 1) - slot_bound(s_slot));
        r->smid = smid_u32();
        r->tag = p.timing_tag;
      }
      int32_t* done = p.slot_claims + kMaxSlots;
      if (atomicAdd(done, 1) == (int)gridDim.x * kDecodeWarps - 1) {
        for (int i = 0; i < p.n_slots; ++i) p.slot_claims[i] = 0;
        *done = 0;
      }
    }
  };
  const bool slot_ok = !(weighted && s_slot < 0);  // always (one CTA per slot)
  auto cost_pref = [&](int b) -> long long { return (long long)s_pref[b] + (long long)kRowCostUnits * s_rpref[b]; };
  // Cost at which row group mg of kv head h of sequence b starts.
  auto row_cost_start = [&](int b, int h, int mg) -> long long {
    const int S = (s_pref[b + 1] - s_pref[b]) / p.Hkv;
    const int NR = (s_rpref[b + 1] - s_rpref[b]) / p.Hkv;
    long long x = cost_pref(b) + (long long)h * (S + (long long)kRowCostUnits * NR);
    for (int m = 0; m < mg; ++m) {
      const int n = units_of(b, m);
      if (n > 0) x += n + kRowCostUnits;
    }
    return x;
  };
  // The first flat unit whose cost position is at least x (W when none).
  auto unit_at_cost = [&](long long x) -> long long {
    if (x >= C) return W;
    int lo = 0, hi = B - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (cost_pref(mid) <= x)
        lo = mid;
      else
        hi = mid - 1;
    }
    // lo is the last sequence whose cost starts at or before x: it has units
    const int S = (s_pref[lo + 1] - s_pref[lo]) / p.Hkv;
    const int NR = (s_rpref[lo + 1] - s_rpref[lo]) / p.Hkv;
    const long long Sc = S + (long long)kRowCostUnits * NR;
    const long long off = x - cost_pref(lo);
    const int h = (int)(off / Sc);
    long long o = off - (long long)h * Sc;
    long long f = s_pref[lo] + (long long)h * S;
    for (int mg = 0; mg < p.NMG; ++mg) {
      const int n = units_of(lo, mg);
      if (n == 0) continue;
      if (o < n + kRowCostUnits) return f + (o > kRowCostUnits ? o - kRowCostUnits : 0);
      o -= n + kRowCostUnits;
      f += n;
    }
    return f;
  };
  const long long ws = slot_ok ? unit_at_cost(warp_start(gw)) : 0;
  const long long we = slot_ok ? unit_at_cost(warp_start(gw + 1)) : 0;
  const bool has_work = slot_ok && W > 0 && gw < nw_eff && ws < we;

  // Locate the first unit of this warp's slice.
  // Flat order: sequence, then kv head, then row group, then unit; a sequence
  // spans Hkv * S_b units with S_b the units of its row groups.
  Cursor start = {0, 0, 0, 0, 0};
  if (has_work) {
    int lo = 0, hi = B - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if ((long long)s_pref[mid] <= ws)
        lo = mid;
      else
        hi = mid - 1;
    }
    start.b = lo;
    const int S = (s_pref[lo + 1] - s_pref[lo]) / p.Hkv;
    int off = (int)(ws - s_pref[lo]);
    start.h = off / S;
    off -= start.h * S;
    start.mg = 0;
    while (true) {
      const int n = units_of(lo, start.mg);
      if (off < n) {
        start.n = n;
        break;
      }
      off -= n;
      ++start.mg;
    }
    start.u = off;
  }
  auto advance = [&](Cursor& c) {
    if (++c.u < c.n) return;
    c.u = 0;
    do {
      if (++c.mg == p.NMG) {
        c.mg = 0;
        if (++c.h == p.Hkv) {
          c.h = 0;
          if (++c.b >= B) return;
        }
      }
      c.n = units_of(c.b, c.mg);
    } while (c.n == 0);
  };

  const uint32_t my_ring = ring_addr + (uint32_t)(warp * stages) * STAGE_BYTES;
  const uint32_t my_bars = smem_addr(&bars[warp * stages]);

  // ---- producer (lane 0 issues; the warp shares the block-table window) ----
  Cursor pc = start;
  long long pf = ws;
  int win_b = -1, win_base = 0, win_val = -1;
  const int bs = p.bs;

  // Keeps block-table entries [win_base, win_base + 32) of sequence win_b in
  // the warp's lanes; reloads (one coalesced load) when lb .. lb+need-1 leave it.
  auto ensure_window = [&](int b, int lb, int need) {
    if (b != win_b || lb < win_base || lb + need > win_base + 32) {
      win_b = b;
      win_base = lb;
      const int e = lb + lane;
      win_val = (e < p.max_blocks) ? __ldg(&p.block_tables[(long long)b * p.bt_stride + e]) : -1;
    }
  };

  // Cascade: when the last unit of a row group is issued, pull the group's
  // prefix state (m, l and the unnormalised accumulator, which the prefix
  // kernel left) into L2, so the fold at the row end does not wait on HBM.
  // Lane pairs take one row each, a half-row of the accumulator per lane.
  auto prefetch_prefix_state = [&](int b, int h, int mg) {
    const int qr = mg * 16 + (lane >> 1);
    if (qr < p.GQ) {
      const int t = qr / p.G, g = qr - t * p.G;
      const long long ridx = ((long long)b * p.Hq + h * p.G + g) * p.q_len + t;
      const float* a = p.pre_acc + ridx * D + (lane & 1) * (D / 2);
#pragma unroll
      for (int c = 0; c < D / 2; c += 32) prefetch_l2(a + c);
      if ((lane & 1) == 0) prefetch_l2(&p.pre_ml[ridx]);
    }
  };

  // The K/V stream is read once: evict-first keeps it from pushing the query
  // rows, partial states, prefix states and tables out of L2.
  const uint64_t kv_policy = l2_policy_evict_first();
  auto issue = [&](int slot) {
    const int h = pc.h;
    if constexpr (cascade) {
      if (pc.u + 1 == pc.n) prefetch_prefix_state(pc.b, h, pc.mg);
    }
    const uint32_t stage = my_ring + (uint32_t)slot * STAGE_BYTES;
    const uint32_t bar = my_bars + (uint32_t)slot * 8u;
    const int tok0 = (pc.u + (cascade ? s_u0[pc.b] : 0)) * kUnitTokens;
    if (bs >= kUnitTokens) {
      const int lb = tok0 / bs;
      const int y = tok0 - lb * bs;
      ensure_window(pc.b, lb, 1);
      const int phys = __shfl_sync(0xffffffffu, win_val, lb - win_base);
      if (lane == 0) {
        if (phys < 0 || phys >= p.num_blocks) raise_flag(p.status, PA_DEVERR_BLOCK_ID_RANGE);
        mbar_arrive_expect_tx(bar, STAGE_BYTES);
#pragma unroll
        for (int hf = 0; hf < HALVES; ++hf)
          tma_load_4d_policy(stage + hf * 2048u, &tmk, bar, hf * 64, y, h, phys, kv_policy);
#pragma unroll
        for (int hf = 0; hf < HALVES; ++hf)
          tma_load_4d_policy(stage + TILE_BYTES + hf * 2048u, &tmv, bar, hf * 64, y, h, phys, kv_policy);
      }
    } else {
      // Block size 8: two blocks per unit; a block past the sequence end is not loaded.
      const int L = s_lens[pc.b];
      const int lb0 = tok0 / bs;
      ensure_window(pc.b, lb0, 2);
      const int phys0 = __shfl_sync(0xffffffffu, win_val, lb0 - win_base);
      const int phys1 = __shfl_sync(0xffffffffu, win_val, lb0 + 1 - win_base);
      if (lane == 0) {
        const bool need1 = (lb0 + 1) * bs < L;
        const uint32_t box_bytes = (uint32_t)bs * 128u;
        const uint32_t nbox = (need1 ? 2u : 1u) * HALVES * 2u;
        if (phys0 < 0 || phys0 >= p.num_blocks || (need1 && (phys1 < 0 || phys1 >= p.num_blocks)))
          raise_flag(p.status, PA_DEVERR_BLOCK_ID_RANGE);
        mbar_arrive_expect_tx(bar, nbox * box_bytes);
        for (int j = 0; j < (need1 ? 2 : 1); ++j) {
          const int phys = j ? phys1 : phys0;
#pragma unroll
          for (int hf = 0; hf < HALVES; ++hf) {
            tma_load_4d_policy(stage + hf * 2048u + j * box_bytes, &tmk, bar, hf * 64, 0, h, phys, kv_policy);
            tma_load_4d_policy(stage + TILE_BYTES + hf * 2048u + j * box_bytes, &tmv, bar, hf * 64, 0, h,
                               phys, kv_policy);
          }
        }
      }
    }
  };

  if (has_work) {
    const int tok0 = (start.u + (cascade ? s_u0[start.b] : 0)) * kUnitTokens;
    ensure_window(start.b, tok0 / bs, bs >= kUnitTokens ? 1 : 2);
  }

  // Everything below reads the K/V cache, which the previous kernel may write
  // (and, under the cascade, the prefix states the previous kernel leaves).
  pdl_wait_previous();
  if constexpr (cascade) fill_empty_rows();
  if (!slot_ok) {  // leave the work undone and say so
    if (lane == 0) raise_flag(p.status, PA_DEVERR_WAIT_TIMEOUT);
    leave_weighted();
    finish_warp();
    return;
  }
  if (weighted && lane == 0) atomicMin(&s_t0, (unsigned long long)global_ns());
  if (!has_work) {
    leave_weighted();
    finish_warp();
    return;
  }

  for (int s = 0; s < stages && pf < we; ++s) {
    issue(s);
    advance(pc);
    ++pf;
  }

  // ---- consumer ----
  const int qrow0 = lane >> 2;  // rows qrow0 and qrow0 + 8 of the m16 tile
  const int quad = lane & 3;
  const int slot_floats = p.slot_rows * (2 + D);

  Cursor cc = start;
  long long cf = ws;
  int slot = 0;
  uint32_t phase = 0;

  uint32_t qa[KSTEPS][4];
  float o_acc[NDT][4];
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  int lim0 = 0, lim1 = 0;  // last attendable token of rows qrow0 / qrow0 + 8
  int mask_from = 0;       // units ending past this position need the causal mask
  bool piece_first = true, piece_from_row_start = false;

  while (cf < we) {
    const int b = cc.b;
    const int h = cc.h;
    const int mg = cc.mg;
    const int L = s_lens[b];

    if (cc.u == 0 || cf == ws) {
      // Begin a piece: load the packed query tile of (b, h, m-group) as A fragments.
      piece_first = (cf == ws);
      piece_from_row_start = (cc.u == 0);
      mask_from = L - p.q_len + (16 * mg) / p.G;  // the group's earliest row's limit
      const int qr0 = mg * 16 + qrow0;
      const int qr1 = qr0 + 8;
      const T* qp0 = nullptr;
      const T* qp1 = nullptr;
      lim0 = L - 1;
      lim1 = L - 1;
      if (qr0 < p.GQ) {
        const int t = qr0 / p.G, g = qr0 - (qr0 / p.G) * p.G;
        qp0 = static_cast<const T*>(p.q) + (long long)b * p.q_sb +
              (long long)(h * p.G + g) * p.q_sh + (long long)t * p.q_st;
        lim0 = L - p.q_len + t;
      }
      if (qr1 < p.GQ) {
        const int t = qr1 / p.G, g = qr1 - (qr1 / p.G) * p.G;
        qp1 = static_cast<const T*>(p.q) + (long long)b * p.q_sb +
              (long long)(h * p.G + g) * p.q_sh + (long long)t * p.q_st;
        lim1 = L - p.q_len + t;
      }
      load_query_frags<T, D>(qa, qp0, qp1, quad, p.Dv);
#pragma unroll
      for (int nd = 0; nd < NDT; ++nd) {
        o_acc[nd][0] = o_acc[nd][1] = o_acc[nd][2] = o_acc[nd][3] = 0.f;
      }
      m0 = m1 = -INFINITY;
      l0 = l1 = 0.f;
    }

    // ---- wait for this unit's K/V tiles ----
    const uint32_t bar = my_bars + (uint32_t)slot * 8u;
    if (!mbar_test_then_wait(bar, (phase >> slot) & 1u)) {
      if (lane == 0) raise_flag(p.status, PA_DEVERR_WAIT_TIMEOUT);
      // Drain this warp's copies still in flight (bounded), then leave.
      int s = slot;
      for (long long k = cf; k < pf; ++k) {
        mbar_wait_bounded(my_bars + (uint32_t)s * 8u, (phase >> s) & 1u);
        s = (s + 1 == stages) ? 0 : s + 1;
      }
      leave_weighted();
      finish_warp();
      return;
    }
    phase ^= (1u << slot);

    const uint32_t kbase = my_ring + (uint32_t)slot * STAGE_BYTES;
    const uint32_t vbase = kbase + TILE_BYTES;

    // ---- QK^T, masked online softmax, PV on tensor cores ----
    attend_unit<T, D>(kbase, vbase, qa, o_acc, m0, m1, l0, l1, (cc.u + (cascade ? s_u0[b] : 0)) * kUnitTokens, L,
                      lim0, lim1, mask_from, p.scale_log2, lane);

    // ---- refill this slot with the unit `stages` ahead ----
    __syncwarp();
    if (pf < we) {
      fence_proxy_async_smem();
      issue(slot);
      advance(pc);
      ++pf;
    }

    // ---- end of a piece: write the output or a partial and merge ----
    const bool row_end = (cc.u + 1 == cc.n);
    if (row_end || cf + 1 == we) {
      float lt0 = l0 + __shfl_xor_sync(0xffffffffu, l0, 1);
      float lt1 = l1 + __shfl_xor_sync(0xffffffffu, l1, 1);
      lt0 += __shfl_xor_sync(0xffffffffu, lt0, 2);
      lt1 += __shfl_xor_sync(0xffffffffu, lt1, 2);
      const int rows_here = min(16, p.GQ - mg * 16);
      const bool r0_ok = qrow0 < rows_here;
      const bool r1_ok = qrow0 + 8 < rows_here;
      // Normalise and store this thread's two rows of the row group from a
      // complete (m, l, acc) state in the MMA fragment layout: to every
      // destination under the fused gather, after folding the prefix state in
      // under the cascade.
      auto finalize_rows = [&](float mm0, float mm1, float ll0, float ll1) {
        const int qa0 = mg * 16 + qrow0, qa1 = qa0 + 8;
        T* op0 = r0_ok ? out_row(0, b, h * p.G + qa0 % p.G, qa0 / p.G) : nullptr;
        T* op1 = r1_ok ? out_row(0, b, h * p.G + qa1 % p.G, qa1 / p.G) : nullptr;
        if constexpr (gather) {
          for (int dst = 0; dst < n_dst; ++dst)
            store_rows<T, D>(r0_ok ? out_row(dst, b, h * p.G + qa0 % p.G, qa0 / p.G) : nullptr,
                             r1_ok ? out_row(dst, b, h * p.G + qa1 % p.G, qa1 / p.G) : nullptr, o_acc, ll0, ll1,
                             quad, p.Dv);
        } else if (cascade && s_u0[b] > 0) {
          const long long rb = (long long)b * p.Hq + h * p.G;
          const long long ridx0 = (rb + qa0 % p.G) * p.q_len + qa0 / p.G;
          const long long ridx1 = (rb + qa1 % p.G) * p.q_len + qa1 / p.G;
          store_rows_folded<T, D>(op0, op1, o_acc, mm0, mm1, ll0, ll1, ridx0, ridx1, p, quad);
        } else {
          store_rows<T, D>(op0, op1, o_acc, ll0, ll1, quad, p.Dv);
        }
      };
      if (row_end && piece_from_row_start) {
        // The whole row is in this piece: normalise and store.
        finalize_rows(m0, m1, lt0, lt1);
      } else {
        // Partial: (m, l, acc) to this warp's slot, then count the arrival.
        const int slot_idx = 2 * gw + (piece_first ? 0 : 1);
        float* sl = p.partials + (long long)slot_idx * slot_floats;
        if (quad == 0) {
          if (r0_ok) {
            sl[qrow0] = m0;
            sl[p.slot_rows + qrow0] = lt0;
          }
          if (r1_ok) {
            sl[qrow0 + 8] = m1;
            sl[p.slot_rows + qrow0 + 8] = lt1;
          }
        }
        float* so = sl + 2 * p.slot_rows;
#pragma unroll
        for (int nd = 0; nd < NDT; ++nd) {
          const int d = nd * 8 + 2 * quad;
          if (r0_ok)
            *reinterpret_cast<float2*>(so + qrow0 * D + d) = make_float2(o_acc[nd][0], o_acc[nd][1]);
          if (r1_ok)
            *reinterpret_cast<float2*>(so + (qrow0 + 8) * D + d) =
                make_float2(o_acc[nd][2], o_acc[nd][3]);
        }
        __threadfence();
        __syncwarp();
        const long long row_start = cf - cc.u;
        const long long row_cost = row_cost_start(b, h, mg) + kRowCostUnits;  // cost position of its unit 0
        const int gw1 = warp_at_cost(row_cost);
        const int gw2 = warp_at_cost(row_cost + cc.n - 1);
        const int npieces = gw2 - gw1 + 1;
        // A split row's counter is indexed by the warp that holds its last unit:
        // that warp starts inside the row, so no other split row ends there.
        // The counter region thus depends only on the grid, not on the batch.
        const int row_id = gw2;
        int old = 0;
        if (lane == 0) old = atomicAdd(&p.counters[row_id], 1);
        old = __shfl_sync(0xffffffffu, old, 0);
        if (old == npieces - 1) {
          // Last arrival: log-sum-exp merge of all pieces of this row.
          __threadfence();
          const bool gw1_first = unit_at_cost(warp_start(gw1)) == row_start;
          auto slot_ptr = [&](int i) -> const float* {
            const int g2 = gw1 + i;
            const int si = (i == 0 && !gw1_first) ? 2 * g2 + 1 : 2 * g2;
            return p.partials + (long long)si * slot_floats;
          };
          if (npieces <= kFragMergePieces) {
            // Few pieces: merge in the MMA fragment layout (each thread its two
            // rows' columns), every piece's loads in flight together, in piece
            // order -- the result does not depend on which warp merges.  The
            // merged state then goes out like a whole row.
            float pm0[kFragMergePieces], pm1[kFragMergePieces], pl0[kFragMergePieces], pl1[kFragMergePieces];
            float M0 = -INFINITY, M1 = -INFINITY;
#pragma unroll
            for (int i = 0; i < kFragMergePieces; ++i) {
              pm0[i] = pm1[i] = -INFINITY;
              pl0[i] = pl1[i] = 0.f;
              if (i < npieces) {
                const float* ps = slot_ptr(i);
                if (r0_ok) {
                  pm0[i] = __ldcg(ps + qrow0);
                  pl0[i] = __ldcg(ps + p.slot_rows + qrow0);
                }
                if (r1_ok) {
                  pm1[i] = __ldcg(ps + qrow0 + 8);
                  pl1[i] = __ldcg(ps + p.slot_rows + qrow0 + 8);
                }
              }
              M0 = fmaxf(M0, pm0[i]);
              M1 = fmaxf(M1, pm1[i]);
            }
            const float base0 = (M0 == -INFINITY) ? 0.f : M0;
            const float base1 = (M1 == -INFINITY) ? 0.f : M1;
            float L0 = 0.f, L1 = 0.f;
#pragma unroll
            for (int nd = 0; nd < NDT; ++nd) o_acc[nd][0] = o_acc[nd][1] = o_acc[nd][2] = o_acc[nd][3] = 0.f;
#pragma unroll
            for (int i = 0; i < kFragMergePieces; ++i) {
              if (i < npieces) {
                const float w0 = ex2(pm0[i] - base0), w1 = ex2(pm1[i] - base1);
                L0 = fmaf(w0, pl0[i], L0);
                L1 = fmaf(w1, pl1[i], L1);
                const float* so = slot_ptr(i) + 2 * p.slot_rows;
#pragma unroll
                for (int nd = 0; nd < NDT; ++nd) {
                  const int d = nd * 8 + 2 * quad;
                  const float2 a0 = r0_ok ? __ldcg(reinterpret_cast<const float2*>(so + qrow0 * D + d))
                                          : make_float2(0.f, 0.f);
                  const float2 a1 = r1_ok ? __ldcg(reinterpret_cast<const float2*>(so + (qrow0 + 8) * D + d))
                                          : make_float2(0.f, 0.f);
                  o_acc[nd][0] = fmaf(w0, a0.x, o_acc[nd][0]);
                  o_acc[nd][1] = fmaf(w0, a0.y, o_acc[nd][1]);
                  o_acc[nd][2] = fmaf(w1, a1.x, o_acc[nd][2]);
                  o_acc[nd][3] = fmaf(w1, a1.y, o_acc[nd][3]);
                }
              }
            }
            finalize_rows(M0, M1, L0, L1);
            if (lane == 0) atomicExch(&p.counters[row_id], 0);
          } else {
          // Many pieces: lanes span the pieces for the max and the weights;
          // each piece's partial accumulators are then read for a few rows at
          // a time, all loads of a piece in flight together.
          constexpr int RG = DPL >= 4 ? 4 : 8;  // rows merged per pass (register budget)
          for (int rg = 0; rg < rows_here; rg += RG) {
            float M[RG], lsum[RG], acc[RG][DPL];
#pragma unroll
            for (int r = 0; r < RG; ++r) {
              M[r] = -INFINITY;
              lsum[r] = 0.f;
#pragma unroll
              for (int k = 0; k < DPL; ++k) acc[r][k] = 0.f;
            }
            for (int i = lane; i < npieces; i += 32) {
              const float* ps = slot_ptr(i);
#pragma unroll
              for (int r = 0; r < RG; ++r)
                if (rg + r < rows_here) M[r] = fmaxf(M[r], __ldcg(ps + rg + r));
            }
#pragma unroll
            for (int r = 0; r < RG; ++r) {
#pragma unroll
              for (int o = 16; o > 0; o >>= 1) M[r] = fmaxf(M[r], __shfl_xor_sync(0xffffffffu, M[r], o));
              if (M[r] == -INFINITY) M[r] = 0.f;  // exponent base of an all-empty row
            }
            for (int i0 = 0; i0 < npieces; i0 += 32) {
              float wgt[RG];
              const int i = i0 + lane;
              if (i < npieces) {
                const float* ps = slot_ptr(i);
#pragma unroll
                for (int r = 0; r < RG; ++r) {
                  wgt[r] = (rg + r < rows_here) ? ex2(__ldcg(ps + rg + r) - M[r]) : 0.f;
                  if (rg + r < rows_here) lsum[r] += wgt[r] * __ldcg(ps + p.slot_rows + rg + r);
                }
              } else {
#pragma unroll
                for (int r = 0; r < RG; ++r) wgt[r] = 0.f;
              }
              const int cnt = min(32, npieces - i0);
#pragma unroll 2
              for (int j = 0; j < cnt; ++j) {
                const float* po = slot_ptr(i0 + j) + 2 * p.slot_rows + rg * D;
                float v[RG][DPL];
#pragma unroll
                for (int r = 0; r < RG; ++r)
#pragma unroll
                  for (int k = 0; k < DPL; ++k)
                    v[r][k] = (rg + r < rows_here) ? __ldcg(po + r * D + lane + 32 * k) : 0.f;
#pragma unroll
                for (int r = 0; r < RG; ++r) {
                  const float wr = __shfl_sync(0xffffffffu, wgt[r], j);
#pragma unroll
                  for (int k = 0; k < DPL; ++k) acc[r][k] = fmaf(wr, v[r][k], acc[r][k]);
                }
              }
            }
#pragma unroll
            for (int r = 0; r < RG; ++r) {
#pragma unroll
              for (int o = 16; o > 0; o >>= 1) lsum[r] += __shfl_xor_sync(0xffffffffu, lsum[r], o);
              if (rg + r < rows_here) {
                const int qr = mg * 16 + rg + r;
                const int t = qr / p.G, g = qr - (qr / p.G) * p.G;
                if (cascade && s_u0[b] > 0) {
                  // fold the row's merged prefix state (loads issued together)
                  const long long ridx = ((long long)b * p.Hq + h * p.G + g) * p.q_len + t;
                  const float2 ml = __ldcg(&p.pre_ml[ridx]);
                  float pa[DPL];
#pragma unroll
                  for (int k = 0; k < DPL; ++k) pa[k] = __ldcg(p.pre_acc + ridx * D + lane + 32 * k);
                  const float M2 = fmaxf(M[r], ml.x);
                  const float c = ex2(M[r] - M2), w = ex2(ml.x - M2);
                  lsum[r] = fmaf(lsum[r], c, w * ml.y);
#pragma unroll
                  for (int k = 0; k < DPL; ++k) acc[r][k] = fmaf(acc[r][k], c, w * pa[k]);
                }
                const float inv = lsum[r] > 0.f ? 1.f / lsum[r] : 0.f;
                for (int dst = 0; dst < n_dst; ++dst) {
                  T* op = out_row(dst, b, h * p.G + g, t);
#pragma unroll
                  for (int k = 0; k < DPL; ++k)
                    if (lane + 32 * k < p.Dv) op[lane + 32 * k] = from_float<T>(acc[r][k] * inv);
                }
              }
            }
          }
          if (lane == 0) atomicExch(&p.counters[row_id], 0);
          }
        }
      }
    }

    advance(cc);
    ++cf;
    slot = (slot + 1 == stages) ? 0 : slot + 1;
  }
  leave_weighted();
  finish_warp();
}

size_t decode_mma_smem_bytes(int D, int B, int stages, bool cascade) {
  const size_t stage_bytes = 2u * 16u * (size_t)D * 2u;
  return 1024 + (size_t)kDecodeWarps * stages * stage_bytes + (size_t)kDecodeWarps * stages * 8 +
         (size_t)((cascade ? 4 : 3) * B + 2) * 4;
}

template <typename T, int D, int kMode>
static cudaError_t launch_mma_impl(const DecodeParams& p, const CUtensorMap& tmk,
                                   const CUtensorMap& tmv, int grid, size_t smem, bool pdl,
                                   cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(kDecodeWarps * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = pdl ? attr : nullptr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, decode_mma_kernel<T, D, kMode>, tmk, tmv, p);
}

template <int kMode>
static cudaError_t launch_mma(const DecodeParams& p, const CUtensorMap& tmk, const CUtensorMap& tmv, int dtype,
                              int grid, size_t smem, bool pdl, cudaStream_t stream) {
  if (dtype == PA_DTYPE_BFLOAT16) {
    if (p.D == 128) return launch_mma_impl<__nv_bfloat16, 128, kMode>(p, tmk, tmv, grid, smem, pdl, stream);
    if (p.D == 64) return launch_mma_impl<__nv_bfloat16, 64, kMode>(p, tmk, tmv, grid, smem, pdl, stream);
  } else if (dtype == PA_DTYPE_FLOAT16) {
    if (p.D == 128) return launch_mma_impl<__half, 128, kMode>(p, tmk, tmv, grid, smem, pdl, stream);
    if (p.D == 64) return launch_mma_impl<__half, 64, kMode>(p, tmk, tmv, grid, smem, pdl, stream);
  }
  return cudaErrorInvalidValue;
}

cudaError_t launch_decode_mma(const DecodeParams& p, const CUtensorMap& tmk, const CUtensorMap& tmv,
                              int dtype, int grid, size_t smem, bool pdl, cudaStream_t stream) {
  if (p.out_ranks != nullptr) return launch_mma<2>(p, tmk, tmv, dtype, grid, smem, pdl, stream);
  if (p.seq_group != nullptr) return launch_mma<1>(p, tmk, tmv, dtype, grid, smem, pdl, stream);
  return launch_mma<0>(p, tmk, tmv, dtype, grid, smem, pdl, stream);
}

template <int kMode>
static const void* decode_fn(int dtype, int D) {
  if (dtype == PA_DTYPE_BFLOAT16)
    return D == 128 ? (const void*)decode_mma_kernel<__nv_bfloat16, 128, kMode>
                    : (const void*)decode_mma_kernel<__nv_bfloat16, 64, kMode>;
  return D == 128 ? (const void*)decode_mma_kernel<__half, 128, kMode>
                  : (const void*)decode_mma_kernel<__half, 64, kMode>;
}

cudaError_t decode_mma_prepare(int dtype, int D, size_t smem) {
  const void* fns[3] = {decode_fn<0>(dtype, D), decode_fn<1>(dtype, D), decode_fn<2>(dtype, D)};
  for (const void* fn : fns) {
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

}  // namespace pa
