// Shared pieces of the SGMV kernels: kernel arguments, the per-CTA copy of
// the slot table and the walk over a CTA's share of the slot-ordered token
// list.
//
// The device segment table (slot_start / token_index, built by segments.cuh)
// lists the active tokens grouped by slot; the kernels process it in items:
// runs of at most kItemTokens tokens of one slot, so that one slot's LoRA
// weights serve the whole item.  The token-split kernels give each CTA a
// contiguous range of tokens (TokenWork).
#pragma once

#include "common.cuh"

namespace plora {

constexpr int kItemTokens = 128;       // tokens per item
constexpr int kFastPathMaxSlots = 1024;  // slot-count limit of the mma kernels (table in smem)

struct SegTable {
  const int32_t* slot_start;   // (num_slots + 1)
  const int32_t* token_index;  // (>= slot_start[num_slots])
  int32_t num_slots;
};

struct ShrinkArgs {
  const uint8_t* x;   // (tokens, K)
  const uint8_t* a;   // (NS, K, R)   (CUDA-core path; the mma path reads it by TMA)
  uint8_t* tmp;       // (tokens, R)
  const int32_t* ranks;
  SegTable seg;
  int32_t K, R, stack_num;
};

struct ExpandArgs {
  const uint8_t* tmp;  // (tokens, R)
  const uint8_t* b;    // (NS, R, N)  (CUDA-core path)
  uint8_t* y;          // (tokens, N)
  const int32_t* ranks;
  const float* scales;
  SegTable seg;
  int32_t R, N;
};

// Per-slot metadata staged in shared memory once per CTA (slot_start, ranks
// and, for the expand, scales), so the schedule never waits on global loads.
struct SlotTab {
  const int32_t* ss;  // (num_slots + 1) slot_start
  const int32_t* rk;  // (num_slots) ranks of this module
  const float* sc;    // (num_slots) scales (expand only)
  int ns;
};

// Copies the table into `dst` (all threads of the CTA; caller syncs).
__device__ __forceinline__ SlotTab stage_slot_tab(const SegTable& t, const int32_t* ranks,
                                                  const float* scales, int32_t* dst) {
  const int ns = t.num_slots;
  int32_t* ss = dst;
  int32_t* rk = dst + ns + 1;
  float* sc = reinterpret_cast<float*>(dst + 2 * ns + 1);
  for (int i = threadIdx.x; i <= ns; i += blockDim.x) ss[i] = ld_cg_i32(t.slot_start + i);
  for (int i = threadIdx.x; i < ns; i += blockDim.x) {
    rk[i] = __ldg(ranks + i);
    sc[i] = scales ? __ldg(scales + i) : 0.f;
  }
  return SlotTab{ss, rk, sc, ns};
}

// Items: maximal runs of <= kItemTokens tokens of one slot inside the CTA's
// contiguous share [p, end) of the slot-ordered token list.
struct SlotItems {
  int64_t p, end;
  int slot;
  __device__ void init(const SlotTab& t, int64_t b, int64_t e) {
    p = b;
    end = e;
    slot = (b < e) ? slot_of_position(t.ss, t.ns, b) : 0;
  }
  __device__ bool next(const SlotTab& t, int& s, int64_t& start, int& cnt) {
    if (p >= end) return false;
    while ((int64_t)t.ss[slot + 1] <= p) ++slot;
    const int64_t lim = min(end, (int64_t)t.ss[slot + 1]);
    cnt = (int)min(lim - p, (int64_t)kItemTokens);
    s = slot;
    start = p;
    p += cnt;
    return true;
  }
};

// ------------------------------------------------------------------ work split
// One piece of a CTA's work: tokens [start, start + cnt) of `slot`, weight
// windows [w_lo, w_hi].
struct Work {
  int64_t start;
  int slot, cnt, w_lo, w_hi;
};

// Token split (batches of many tokens): the CTA's contiguous share [b, e) of
// the slot-ordered token list, cut into items; every item covers all `nwin`
// weight windows of its slot.
struct TokenWork {
  SlotItems it;
  int nwin;
  __device__ void init(const SlotTab& t, int64_t b, int64_t e, int nw) {
    it.init(t, b, e);
    nwin = nw;
  }
  __device__ __forceinline__ bool next(const SlotTab& t, Work& w) {
    int s, cnt;
    int64_t start;
    while (it.next(t, s, start, cnt))
      if (t.rk[s] > 0) {
        w.start = start;
        w.slot = s;
        w.cnt = cnt;
        w.w_lo = 0;
        w.w_hi = nwin - 1;
        return true;
      }
    return false;
  }
};

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~(uintptr_t)1023);
}

}  // namespace plora
