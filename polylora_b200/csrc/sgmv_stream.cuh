// Rank-16 SGMV shrink and expand for batches of many tokens: the slot's LoRA
// weights held in registers, token rows moved by bulk copies (shrink) or
// reduced into y by the L2 (expand).
//
// Both kernels move bytes and do almost no arithmetic (10.7 flop per byte at
// rank 16); their speed is set by how many bytes each SM keeps in flight and
// by how little waiting sits between a copy landing and the next one being
// issued.
//  * At rank 16 a slot's LoRA-A (K x 16) or LoRA-B (16 x N) is 128 KB for K
//    or N = 4096.  Split over 16 warps that is 8 KB per warp, 64 registers per
//    lane in mma fragment layout.
//  * shrink: token rows travel by one plain `cp.async.bulk` per row
//    (K * 2 bytes) into a ring of shared-memory stages of 8 rows, at a
//    (K * 2 + 16)-byte pitch so that ldmatrix over eight rows hits eight bank
//    groups.  The ring carries token rows only, refilled by a producer warp;
//    each consumer warp loads its slice of LoRA-A straight into registers
//    (two 8-byte loads per k16 step, turned into the mma layout by
//    movmatrix.trans; see shrink_rank_of_row), so the first token rows are
//    requested at launch, beside the weights, and a change of slot costs one
//    L2 round trip (the slot's rows are prefetched into L2 when the producer
//    first meets it) instead of 128 KB of ring stages.  Warp w owns K rows
//    [w K/16, (w + 1) K/16): per stage it
//    multiplies its slice of the 8 rows by its A fragments (mma.sync
//    m16n8k16, D^T = A^T x^T, fp32) and publishes the 16 x 8 partial in
//    shared memory.  Group i's partials are added, in warp order
//    (deterministic), by warp i mod 16 two groups later, which rounds and
//    writes tmp: the reduction is spread over the warps, and by then every
//    warp has long published group i, so the reducer does not wait.
//  * expand: the weights arrive as "weight stages" (LoRA-B rank rows 0-7 and
//    8-15) by bulk copies through a ring of two, and the warps move their
//    column slices into registers with ldmatrix.trans.
//    Warp w owns N columns [w N/16, (w + 1) N/16).  Per group of 8
//    tokens it computes delta = tmp B for its columns (mma.sync with the tmp
//    rows as A fragments; the share's tmp rows are gathered into shared
//    memory by cp.async once, at the start), rounds scale * delta to
//    the activation type, regroups the fragments so that each lane holds 8
//    consecutive columns of one row (stmatrix into a per-warp tile), and
//    adds them to y with `red.global.add.noftz.v4.{bf16x2,f16x2}`: the L2
//    reads y, adds and rounds to nearest, so y never passes through the SM
//    and nothing waits for it; the result is the reference's (round the
//    scaled delta, then the sum) bit for bit.
// The expand's weight stages are refilled by the last of the 16 warps to
// finish with them.  Work split: a CTA per SM takes a contiguous share of the
// slot-ordered token list (its token ids are copied to shared memory once, so
// no global load sits between a stage landing and its refill), cut into
// groups of <= 8 tokens of one slot.  At the start the slot table is read
// first, so that the first weights are requested one global round trip after
// launch.
// Every wait is bounded; after an expiry or an abort the warps leave their
// loops, and thread 0 waits (bounded) for the loads already issued before the
// CTA exits.
//
// Reference semantics: src/polylora/sgmv.py:63-138 (_sgmv_lora_a_kernel) and
// sgmv.py:178-275 (_sgmv_lora_b_kernel).
#pragma once

#include "sgmv_mma.cuh"

namespace plora {

constexpr int kStreamRank = 16;            // the rank tile these kernels serve
constexpr int kStreamWarps = 16;
constexpr int kStreamThreads = kStreamWarps * 32;
constexpr int kStreamMaxStages = 16;
constexpr int kStreamSmemLimit = 232448;   // dynamic shared memory per CTA (227 KB)
constexpr int kStreamMaxDim = 4096;        // K (shrink) / N (expand): 64 fragment registers
constexpr int kStreamGroup = 8;            // tokens per group (the mma's 8-wide half)
constexpr int kStreamWeightParts = 2;      // weight stages per slot
// Token ids of a CTA's share staged in shared memory: calls whose num_tokens
// exceeds this times the SM count use the windowed kernels instead.
constexpr int kStreamMaxShare = 1024;
constexpr int kShrinkPartBufs = 3;                                     // partial buffers in flight
constexpr int kShrinkReduceLag = 2;  // group i is reduced at group i + 2 (< kShrinkPartBufs)
constexpr int kShrinkPartBytes = kStreamWarps * 32 * 16;               // one group's 16 partials
constexpr int kShrinkTmpTileBytes = kStreamWarps * kStreamGroup * kStreamRank * 2;  // per warp: a group's tmp rows
constexpr int kShrinkMetaBytes = 64;  // per partial buffer: slot, token count, start of its group
constexpr int kExpandTmpRowBytes = kStreamRank * 2;                    // one token's tmp row
constexpr int kExpandRegroupBytes = kStreamWarps * kStreamGroup * 64;  // per warp 8 rows x 32 columns

// Shared-memory plan of a stream kernel (host and device alike), offsets from
// the 128-byte aligned base:
//   shrink: [nst token stages][3 partial buffers][tmp tiles][group of each buffer][barriers]
//           [token ids][slot table]
//   expand: [2 weight stages][tmp rows of the share][regroup tiles][barriers][token ids][slot table]
// Barrier area (expand): per weight stage an mbarrier (8 B), a release count
// and the index of the last item loaded (4 B each); then 6 unused mbarrier
// words and the abort flag.  The shrink's is laid out by shrink_bar_bytes.
struct StreamPlan {
  int nst;               // shrink: token stages; expand: weight stages
  uint32_t pitch;        // token / weight row pitch in a stage
  uint32_t stage_bytes;  // 8 rows
  uint32_t aux_off;      // shrink: partial buffers; expand: the share's tmp rows
  uint32_t rg_off;       // regroup tiles (shrink: tmp rows of a group; expand: delta columns)
  uint32_t bar_off, tok_off, tab_off;
  uint32_t smem_bytes;   // dynamic shared memory to request (includes 128 B of alignment slack)
};

__host__ __device__ inline uint32_t stream_bar_bytes(int slots) { return (uint32_t)slots * 16 + 6 * 8 + 16; }
// shrink: per stage a full and an empty mbarrier (16 B) and the last item armed
// (4 B, after the 6 partial barriers), then the abort flag
__host__ __device__ inline uint32_t shrink_bar_bytes(int stages) { return (uint32_t)stages * 20 + 6 * 8 + 16; }

__host__ __device__ inline StreamPlan shrink_stream_plan(int64_t K, int64_t num_slots, int64_t extra_bar_bytes = 0) {
  StreamPlan p;
  p.pitch = (uint32_t)(K * 2 + 16);
  p.stage_bytes = p.pitch * kStreamGroup;
  const int64_t tab = slot_tab_bytes(num_slots);
  const int64_t fixed =
      128 + kShrinkPartBufs * kShrinkPartBytes + kShrinkTmpTileBytes + kShrinkMetaBytes + shrink_bar_bytes(0) +
      extra_bar_bytes + kStreamMaxShare * 4 + tab;
  int64_t nst = (kStreamSmemLimit - fixed) / ((int64_t)p.stage_bytes + 24);
  if (nst > kStreamMaxStages) nst = kStreamMaxStages;
  p.nst = (int)nst;
  p.aux_off = (uint32_t)(nst * p.stage_bytes);
  p.rg_off = p.aux_off + kShrinkPartBufs * kShrinkPartBytes;
  p.bar_off = p.rg_off + kShrinkTmpTileBytes + kShrinkMetaBytes;
  p.tok_off = p.bar_off + shrink_bar_bytes(p.nst) + (uint32_t)extra_bar_bytes;
  p.tab_off = p.tok_off + kStreamMaxShare * 4;
  p.smem_bytes = (uint32_t)(128 + p.tab_off + tab);
  return p;
}

// The fused shrink + expand kernel's expand phase reuses the shrink's shared
// memory once the token ring is idle: two LoRA-B weight stages and the share's
// tmp rows in the ring area, the regroup tiles in the partial buffers, and 2
// full + 2 empty mbarriers and 2 last-armed indices after the shrink's barriers.
struct FusedPlan {
  uint32_t w_pitch = 0, w_stage_bytes = 0;  // weight stage: 8 rows of N values
  uint32_t tmp_off = 0, rg_off = 0, wbar_off = 0;
};
constexpr int kFusedBarBytes = 8 + 2 * 8 + 2 * 8 + 2 * 4;  // alignment pad + barriers + indices

// Plans of the fused kernel for K x N; false when the expand phase does not
// fit the shrink's ring area (then the two kernels run one after the other).
__host__ __device__ inline bool fused_stream_plan(int64_t K, int64_t N, int64_t num_slots, StreamPlan& sp,
                                                  FusedPlan& fp) {
  sp = shrink_stream_plan(K, num_slots, kFusedBarBytes);
  fp.w_pitch = (uint32_t)(N * 2 + 16);
  fp.w_stage_bytes = fp.w_pitch * kStreamGroup;
  fp.tmp_off = 2 * fp.w_stage_bytes;
  fp.rg_off = sp.aux_off;
  fp.wbar_off = (sp.bar_off + shrink_bar_bytes(sp.nst) + 7u) & ~7u;
  return sp.nst >= 2 && (int64_t)fp.tmp_off + kStreamMaxShare * kExpandTmpRowBytes <= (int64_t)sp.nst * sp.stage_bytes &&
         kExpandRegroupBytes <= kShrinkPartBufs * kShrinkPartBytes && fp.wbar_off + 40u <= sp.tok_off &&
         sp.smem_bytes <= (uint32_t)kStreamSmemLimit;
}

__host__ __device__ inline StreamPlan expand_stream_plan(int64_t N, int64_t num_slots) {
  StreamPlan p;
  p.nst = kStreamWeightParts;
  p.pitch = (uint32_t)(N * 2 + 16);
  p.stage_bytes = p.pitch * kStreamGroup;
  p.aux_off = kStreamWeightParts * p.stage_bytes;
  p.rg_off = p.aux_off + kStreamMaxShare * kExpandTmpRowBytes;
  p.bar_off = p.rg_off + kExpandRegroupBytes;
  p.tok_off = p.bar_off + stream_bar_bytes(kStreamWeightParts);
  p.tab_off = p.tok_off + kStreamMaxShare * 4;
  p.smem_bytes = (uint32_t)(128 + p.tab_off + slot_tab_bytes(num_slots));
  return p;
}

// ---------------------------------------------------------------- copies
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// Global -> shared bulk copy (16-byte aligned, size a multiple of 16) completing on `bar`.
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint64_t* bar,
                                          uint64_t pol) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1], %2, [%3], %4;" ::"r"(dst),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(pol)
      : "memory");
}

// Asks the L2 to fetch [src, src + bytes) (16-byte aligned, a multiple of 16);
// nothing waits for it.
__device__ __forceinline__ void prefetch_l2_bulk(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// 8-byte load of data that no kernel writes while this one runs, not kept in L1.
__device__ __forceinline__ uint2 ld_nc_v2(const void* p) {
  uint2 v;
  asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
  return v;
}

// Transposes the 8 x 8 16-bit matrix the warp holds in row layout (lane l:
// row l >> 2, columns 2 (l & 3) and + 1) into the same layout.
__device__ __forceinline__ uint32_t movmatrix_t(uint32_t v) {
  uint32_t d;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(d) : "r"(v));
  return d;
}

__device__ __forceinline__ void cp_async16_cg(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
// The barrier tracks this thread's earlier cp.async copies: its pending count
// rises by one now and falls when they have landed.
__device__ __forceinline__ void cp_async_mbar_arrive(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
      : "memory");
}

// dst[0..7] += v (eight 16-bit values, the sums rounded to nearest by the L2).
template <bool BF16>
__device__ __forceinline__ void red_add_v8(void* dst, const uint32_t (&v)[4]) {
  if constexpr (BF16)
    asm volatile("red.global.add.noftz.v4.bf16x2 [%0], {%1, %2, %3, %4};" ::"l"(dst), "r"(v[0]), "r"(v[1]),
                 "r"(v[2]), "r"(v[3])
                 : "memory");
  else
    asm volatile("red.global.add.noftz.v4.f16x2 [%0], {%1, %2, %3, %4};" ::"l"(dst), "r"(v[0]), "r"(v[1]),
                 "r"(v[2]), "r"(v[3])
                 : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ uint8_t* align128(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 127) & ~(uintptr_t)127);
}

// ---------------------------------------------------------------- items
// Items of a CTA: for every run of tokens of one slot of rank > 0 inside the
// CTA's share of the slot-ordered token list, the slot's two weight stages
// (unless the sequence is made without them), then its groups of <= 8 tokens
// (runs of rank-0 slots are skipped).  Positions are relative to the share's
// start `base`.
struct RingItem {
  int part;  // weight stage 0 / 1, or -1 for a token group
  int slot, cnt, start;
};

struct RingSeq {
  int p, end, slot, wslot, wpart;  // wslot: slot whose weight stages were last emitted
  bool low_half_only;              // slots of rank <= 8 need only weight stage 0 (expand)
  bool weights;                    // false: token groups only
  __device__ void init(const SlotTab& t, int64_t b, int64_t e, bool rank8_one_stage = false,
                       bool with_weights = true) {
    p = 0;
    end = (int)(e - b);
    slot = (b < e) ? slot_of_position(t.ss, t.ns, b) : 0;
    wslot = -1;
    wpart = 0;
    low_half_only = rank8_one_stage;
    weights = with_weights;
  }
  __device__ __forceinline__ bool next(const SlotTab& t, int64_t base, RingItem& it) {
    while (p < end) {
      while ((int64_t)t.ss[slot + 1] <= base + p) ++slot;
      const int lim = (int)min((int64_t)end, (int64_t)t.ss[slot + 1] - base);
      if (t.rk[slot] <= 0) {
        p = lim;
        continue;
      }
      it.slot = slot;
      it.start = p;
      if (weights && slot != wslot) {
        it.part = wpart;
        it.cnt = 0;
        if (++wpart == kStreamWeightParts || (low_half_only && t.rk[slot] <= 8)) {
          wpart = 0;
          wslot = slot;
        }
        return true;
      }
      it.part = -1;
      it.cnt = min(lim - p, kStreamGroup);
      p += it.cnt;
      return true;
    }
    return false;
  }
  // the next item of one kind (weight stages: want_weight; token groups: !want_weight)
  __device__ __forceinline__ bool next_of(const SlotTab& t, int64_t base, RingItem& it, bool want_weight) {
    while (next(t, base, it))
      if ((it.part >= 0) == want_weight) return true;
    return false;
  }
};

// Cost-balanced shares.  A token costs 1 and every run of an active slot
// (rank > 0, at least one token) costs `slot_cost` more: the slot's weights,
// which every CTA whose share reaches into the run loads in full.  In the
// "virtual" coordinate VS_j = slot_start[j] + slot_cost * (active slots before
// j) a slot's weights come first, then its tokens; CTA b of G takes virtual
// [V b / G, V (b + 1) / G), V = total + slot_cost * active slots, and a cut at
// virtual v falls at token position
//   s_J                                  v - VS_J <= slot_cost, J active
//   min(s_J + v - VS_J - slot_cost, s_J+1)  otherwise for an active J
//   min(s_J + v - VS_J, s_J+1)            J inactive
// with J the last slot whose VS_J <= v (a cut inside a slot's weight units
// falls at its first token).  So a share that reaches into one more slot
// holds fewer tokens, and the CTAs finish together.  The cut is monotone in
// v, 0 at v = 0 and total at v = V, so the shares are contiguous and cover
// the list; a share holds at most ceil(V / G) + 1 tokens.
struct StreamCut {
  int J = 0;
  int64_t vs = 0;
  bool act = false;
  __device__ __forceinline__ int64_t position(const SlotTab& t, int64_t v, int64_t slot_cost) const {
    if (J >= t.ns) return t.ss[t.ns];
    const int64_t off = v - vs, s0 = t.ss[J], s1 = t.ss[J + 1];
    if (act) return off <= slot_cost ? s0 : min(s0 + off - slot_cost, s1);
    return min(s0 + off, s1);
  }
};

// [begin, end) of CTA b of G, both cuts found in one walk over the staged slot
// table, 32 slots per step.  `nact` is the number of active slots.
// Warp-collective: every lane returns the share.
__device__ void stream_share(const SlotTab& t, int nact, int b, int G, int64_t slot_cost, int lane, int64_t& begin,
                             int64_t& end) {
  const int64_t V = (int64_t)t.ss[t.ns] + slot_cost * nact;
  const int64_t v0 = V * b / G, v1 = V * (b + 1) / G;
  StreamCut c0, c1;
  int64_t carry = 0;  // active slots before this step's 32
  for (int c = 0; c <= t.ns; c += 32) {
    const int j = c + lane;
    const bool valid = j <= t.ns;
    const bool act = j < t.ns && t.rk[j] > 0 && t.ss[j + 1] > t.ss[j];
    const uint32_t am = __ballot_sync(0xffffffffu, act);
    const int64_t vs = valid ? t.ss[j] + slot_cost * (carry + __popc(am & ((1u << lane) - 1u))) : 0;
    // VS is non-decreasing, so the slots with VS_j <= v are a prefix of the lanes
    const uint32_t le0 = __ballot_sync(0xffffffffu, valid && vs <= v0);
    const uint32_t le1 = __ballot_sync(0xffffffffu, valid && vs <= v1);
    if (le0 != 0u) {
      const int last = 31 - __clz(le0);
      c0.J = c + last;
      c0.vs = __shfl_sync(0xffffffffu, vs, last);
      c0.act = (am >> last) & 1u;
    }
    if (le1 != 0u) {
      const int last = 31 - __clz(le1);
      c1.J = c + last;
      c1.vs = __shfl_sync(0xffffffffu, vs, last);
      c1.act = (am >> last) & 1u;
    }
    if (le1 != 0xffffffffu) break;  // v0 <= v1: both cuts are found
    carry += __popc(am);
  }
  begin = c0.position(t, v0, slot_cost);
  end = c1.position(t, v1, slot_cost);
}

// stage_slot_tab, also counting how many of the slots this thread staged are
// active (rank > 0, at least one token); without scales the table's scale
// column is not written.
__device__ __forceinline__ SlotTab stage_slot_tab_counted(const SegTable& t, const int32_t* ranks, const float* scales,
                                                          int32_t* dst, int& active_mine) {
  const int ns = t.num_slots;
  int32_t* ss = dst;
  int32_t* rk = dst + ns + 1;
  float* sc = reinterpret_cast<float*>(dst + 2 * ns + 1);
  active_mine = 0;
  for (int i = threadIdx.x; i <= ns; i += blockDim.x) {
    const int32_t s0 = ld_cg_i32(t.slot_start + i);
    ss[i] = s0;
    if (i < ns) {
      const int32_t s1 = ld_cg_i32(t.slot_start + i + 1);
      const int32_t r = __ldg(ranks + i);
      rk[i] = r;
      if (scales) sc[i] = __ldg(scales + i);
      active_mine += (r > 0 && s1 > s0) ? 1 : 0;
    }
  }
  return SlotTab{ss, rk, sc, ns};
}

// A ring of `n` stages in shared memory: full barriers, release counts and
// the last item index loaded into each stage.
struct StreamRing {
  uint64_t* full;
  uint32_t* released;  // monotonic; the 16th warp of an item refills the stage
  int32_t* loaded;     // -1: nothing loaded
  int n;
  __device__ void carve(uint8_t* p, int slots) {
    full = reinterpret_cast<uint64_t*>(p);
    released = reinterpret_cast<uint32_t*>(full + slots);
    loaded = reinterpret_cast<int32_t*>(released + slots);
    n = slots;
  }
  __device__ void init() const {  // one thread
    for (int i = 0; i < n; ++i) {
      mbar_init(&full[i], 1);
      released[i] = 0;
      loaded[i] = -1;
    }
  }
  // Counts this warp out of stage s; true (on every lane) for the 16th warp of
  // the item.  Prior shared-memory accesses of the warp are ordered before it.
  __device__ __forceinline__ bool release(int s, int lane) const {
    __syncwarp();
    int last = 0;
    if (lane == 0) {
      __threadfence_block();
      last = (atomicAdd(&released[s], 1u) % kStreamWarps) == kStreamWarps - 1;
      __threadfence_block();
    }
    return __shfl_sync(0xffffffffu, last, 0) != 0;
  }
  // Thread 0 at CTA exit: the last load issued into each stage has landed (it
  // has unless the warps gave up early), so no copy writes freed shared memory.
  __device__ void drain() const {
    for (int s = 0; s < n; ++s)
      if (loaded[s] >= 0) mbar_drain(&full[s], (uint32_t)(loaded[s] / n) & 1u);
  }
};

// Arms stage s of item ii for `bytes` of bulk copies (lane 0 of the issuing warp).
// The stage's earlier readers (ldmatrix) released it before the last of them
// got here, so the copies may overwrite it.
__device__ __forceinline__ void ring_arm(const StreamRing& r, int s, int ii, uint32_t bytes) {
  r.loaded[s] = ii;
  mbar_arrive_expect_tx(&r.full[s], bytes);
}

// Weight stage (whole warp): lanes < 8 copy `len` bytes from src + lane * len
// to dst + lane * dst_stride.
__device__ __forceinline__ void ring_issue_weights(const StreamRing& r, int ii, const uint8_t* src, uint32_t dst,
                                                   uint32_t dst_stride, uint32_t len, uint64_t pol, int lane) {
  const int s = ii % r.n;
  if (lane == 0) ring_arm(r, s, ii, 8 * len);
  __syncwarp();
  if (lane < 8) bulk_load(dst + lane * dst_stride, src + (int64_t)lane * len, len, &r.full[s], pol);
}

// Copies the CTA's token ids [begin, end) into shared memory (all threads; caller syncs).
__device__ __forceinline__ void stream_stage_tokens(const int32_t* token_index, int64_t begin, int64_t end,
                                                    int32_t* dst) {
  for (int64_t i = threadIdx.x; i < end - begin; i += blockDim.x) dst[i] = ld_cg_i32(token_index + begin + i);
}
// The same by one warp, 256 ids per round trip.
__device__ __forceinline__ void stream_stage_tokens_warp(const int32_t* token_index, int64_t begin, int64_t end,
                                                         int32_t* dst, int lane) {
  constexpr int kPerLane = 8;
  const int n = (int)(end - begin);
  for (int c = 0; c < n; c += 32 * kPerLane) {
    int32_t v[kPerLane];
#pragma unroll
    for (int k = 0; k < kPerLane; ++k)
      if (c + k * 32 + lane < n) v[k] = ld_cg_i32(token_index + begin + c + k * 32 + lane);
#pragma unroll
    for (int k = 0; k < kPerLane; ++k)
      if (c + k * 32 + lane < n) dst[c + k * 32 + lane] = v[k];
  }
}

// ============================================================== shrink
// tmp[t, :] = x[t, :] @ A[slot(t)] (rank 16) for the active tokens of the
// table; columns >= min(rank * stack_num, 16) of an active token are written
// as 0, inactive tokens are not written.  K % 512 == 0, K <= 4096.
//
// Roles: warps 0-15 consume token stages; warp 16 stages the share's token
// ids and refills the ring (it waits for a stage's 16 releases on an mbarrier,
// then issues the stage's row copies), so a bulk copy that stalls at issue
// while the copy engine is busy delays no consumer.  Warps 17-19 only make the
// producer a whole warpgroup: the CTA is launched at kShrinkLaunchRegs
// registers a thread and setmaxnreg moves the producer warpgroup's share to
// the consumers (64 fragment registers each).
//
// A fragments from global memory: for its k16 step at row k0, lane (g, t)
// loads ranks 4t .. 4t + 3 of rows k0 + g and k0 + 8 + g (8 bytes each).  The
// low half of the first load is element (g, 2t) of the 8 x 8 block "rows k0 ..
// k0 + 7, ranks 4c + {0, 1} for column pair c" in row layout, the high half
// the same for ranks 4c + {2, 3}; movmatrix.trans turns each into the A^T
// fragment.  So mma row r (r < 8) holds rank shrink_rank_of_row(r) = 4 (r >> 1)
// + (r & 1) and row 8 + r holds that rank + 2; the reduction writes tmp in
// rank order.  A warp's step reads 8 whole 32-byte rows of A (256 contiguous
// bytes) per load instruction.
constexpr int kShrinkThreads = kStreamThreads + 128;  // 16 consumer warps + the producer warpgroup
constexpr int kShrinkLaunchRegs = 96;                 // 5 warps per scheduler partition
constexpr int kShrinkConsumerRegs = 112;
constexpr int kShrinkProducerRegs = 32;
constexpr int kShrinkIdsReady = 1;  // named barrier: the producer has staged the token ids
// Extra cost of a slot's run in a share, in tokens: loading the slot's 128 KB
// of LoRA-A (16 rows' worth of x bytes) and the stall around it.
constexpr int64_t kShrinkSlotCost = 20;
static_assert(kFastPathMaxSlots <= 2 * kShrinkThreads, "a thread stages at most 2 slots");
// per scheduler partition: 4 consumer warps + 1 producer-group warp within the launch's registers
static_assert(4 * kShrinkConsumerRegs + kShrinkProducerRegs <= 5 * kShrinkLaunchRegs, "register split");
static_assert(5 * 32 * kShrinkLaunchRegs <= 16384, "launch registers per partition");

__host__ __device__ constexpr int shrink_rank_of_row(int r) { return 4 * ((r & 7) >> 1) + (r & 1) + 2 * (r >> 3); }

// 16-byte load through L2: for data that other threads of this CTA wrote
// before a barrier.
__device__ __forceinline__ uint4 ld_cg_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.cg.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}

constexpr int kFusedTmpWritten = 2;  // named barrier of the 16 consumer warps (fused kernel)

// The fused kernel's expand phase (consumer warps 0-15): y[t, :] +=
// round(scale * tmp[t, :] @ B[slot(t)]) for the CTA's share, as
// sgmv_expand_stream_kernel computes it, with the weight stages streamed by
// the producer warp (wfull / wempty) and the share's tmp rows gathered from
// global memory, where this CTA's reducers wrote them.  Every consumer warp
// passes both barriers, also after an abort.
template <bool BF16>
__device__ __forceinline__ void fused_expand_phase(const ExpandArgs& args, const FusedPlan& fp, const SlotTab& tab,
                                                   const int32_t* tok_s, int64_t begin, int64_t end, uint32_t stage0,
                                                   volatile int* abort_flag, uint64_t* wfull, uint64_t* wempty,
                                                   uint8_t* smem, int warp, int lane) {
  const int N = args.N;
  const int share = (int)(end - begin);
  uint8_t* tmp_s = smem + fp.tmp_off;
  named_barrier(kFusedTmpWritten, kStreamThreads);  // every group's tmp rows are in global memory
  if (!*abort_flag)
    for (int i = threadIdx.x; i < 2 * share; i += kStreamThreads)
      *reinterpret_cast<uint4*>(tmp_s + i * 16) =
          ld_cg_v4(args.tmp + (int64_t)tok_s[i >> 1] * kExpandTmpRowBytes + (i & 1) * 16);
  named_barrier(kFusedTmpWritten, kStreamThreads);

  const uint32_t row_bytes = (uint32_t)N * 2;
  const int g = lane >> 2;
  const int t = lane & 3;
  const int ncw = N >> 4;   // columns of this warp
  const int nt = ncw >> 3;  // n8 tiles of this warp: a multiple of 4, <= 32
  const int c0w = warp * ncw;
  uint32_t b[32][2];
  const uint32_t w_off = (uint32_t)(lane & 7) * fp.w_pitch + (uint32_t)(c0w + 8 * (lane >> 3)) * 2;
  const uint32_t rg_base = stage0 + fp.rg_off + warp * kStreamGroup * 64;
  const uint32_t rg_st = rg_base + (lane & 7) * 64 + 16 * ((lane >> 3) ^ (((lane & 7) >> 1) & 3));
  const uint32_t rg_ld = rg_base + g * 64 + 16 * (t ^ ((g >> 1) & 3));
  float scale = 0.f;
  int kr = 0;
  RingSeq it;
  it.init(tab, begin, end, true, true);
  int wi = 0;
  RingItem cq;
  while (it.next(tab, begin, cq)) {
    if (cq.part >= 0) {  // weight stage: rank rows 8 part .. of this warp's columns
      const int w = wi & 1;
      if (!mbar_wait_warp(&wfull[w], (uint32_t)(wi / 2) & 1u, abort_flag)) break;
      if (cq.part == 0) {
        scale = tab.sc[cq.slot];
        kr = min(tab.rk[cq.slot], args.R);
      }
      const uint32_t sbase = stage0 + w * fp.w_stage_bytes;
      const bool one_stage = kr <= 8;
#pragma unroll
      for (int i = 0; i < 32; i += 4)
        if (i < nt) {
          uint32_t r[4];
          ldsm_x4_t(sbase + w_off + 16 * i, r);
#pragma unroll
          for (int m = 0; m < 4; ++m) {
            if (cq.part == 0) {
              b[i + m][0] = r[m];
              if (one_stage) b[i + m][1] = 0u;
            } else {
              b[i + m][1] = r[m];
            }
          }
        }
      __syncwarp();
      if (lane == 0) mbar_arrive(&wempty[w]);
      ++wi;
      continue;
    }
    uint32_t fa[4] = {0u, 0u, 0u, 0u};
    const bool vrow = g < cq.cnt;
    int64_t tok = 0;
    if (vrow) {
      const uint32_t* trow = reinterpret_cast<const uint32_t*>(tmp_s + (cq.start + g) * kExpandTmpRowBytes);
      auto ld2 = [&](int k) -> uint32_t {
        if (k >= kr) return 0u;
        const uint32_t v = trow[k >> 1];
        return k + 1 < kr ? v : (v & 0xFFFFu);
      };
      fa[0] = ld2(2 * t);
      fa[2] = ld2(2 * t + 8);
      tok = tok_s[cq.start + g];
    }
    uint8_t* yrow = args.y + tok * row_bytes + (c0w + 8 * t) * 2;
#pragma unroll
    for (int i = 0; i < 32; i += 4)
      if (i < nt) {
        uint32_t d[4];
#pragma unroll
        for (int m = 0; m < 4; ++m) {
          float acc[4] = {0.f, 0.f, 0.f, 0.f};
          mma_16816<BF16>(acc, fa, b[i + m][0], b[i + m][1]);
          d[m] = pack2<BF16>(scale * acc[0], scale * acc[1]);
        }
        stsm_x4(rg_st, d);
        __syncwarp();
        lds_v4(rg_ld, d);
        __syncwarp();
        if (vrow) red_add_v8<BF16>(yrow + 16 * i, d);
      }
  }
}


// kFused: the fused shrink + expand kernel.  After its shrink phase a CTA
// expands its own share: the producer waits until every ring stage has been
// released for the last time and streams the share's LoRA-B weight stages
// into the idle ring (prefetched into L2 while the shrink ran); the consumers
// pass a barrier (every group's tmp rows written by their reducers), gather
// the share's tmp rows into shared memory (they are still in L2) and run the
// expand's group loop (sgmv_expand_stream_kernel).  No grid-wide dependency:
// a CTA's expand phase reads only its own tmp rows, so it starts while other
// CTAs still shrink, and the expand's launch, slot table and token ids are
// not paid twice.
template <bool BF16, bool kFused>
__global__ void __launch_bounds__(kShrinkThreads, 1)
    sgmv_shrink_stream_kernel(const ShrinkArgs args, const StreamPlan plan, const ExpandArgs eargs,
                              const FusedPlan fp) {
  using E = Elem<BF16>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align128(smem_raw);
  const int nst = plan.nst;
  const int K = args.K;
  float* part = reinterpret_cast<float*>(smem + plan.aux_off);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + plan.bar_off);  // [nst] token rows landed
  uint64_t* empty = full + nst;                                         // [nst] 16 consumer warps released
  uint64_t* pfull = empty + nst;              // [3] all 16 partials of the group written
  uint64_t* pempty = pfull + kShrinkPartBufs;  // [3] the group's partials have been read
  int32_t* loaded = reinterpret_cast<int32_t*>(pempty + kShrinkPartBufs);  // [nst] last item armed, -1 none
  volatile int* abort_flag = reinterpret_cast<volatile int*>(loaded + nst);
  int32_t* tok_s = reinterpret_cast<int32_t*>(smem + plan.tok_off);
  int32_t* tab_mem = reinterpret_cast<int32_t*>(smem + plan.tab_off);
  // fused expand phase: [2] weight stage landed, [2] released by the 16 consumers, [2] last item armed
  uint64_t* wfull = reinterpret_cast<uint64_t*>(smem + fp.wbar_off);
  uint64_t* wempty = wfull + 2;
  int32_t* wloaded = reinterpret_cast<int32_t*>(wempty + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  griddep_wait();    // inputs (segment table, x) come from earlier kernels
  griddep_launch();  // the expand may start on SMs this grid releases
  int active_mine;  // active slots among those this thread staged (<= 2)
  const SlotTab tab = stage_slot_tab_counted(args.seg, args.ranks, kFused ? eargs.scales : nullptr, tab_mem,
                                             active_mine);
  if (threadIdx.x == 0) {
    for (int i = 0; i < nst; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kStreamWarps);
      loaded[i] = -1;
    }
    if constexpr (kFused) {
      for (int i = 0; i < 2; ++i) {
        mbar_init(&wfull[i], 1);
        mbar_init(&wempty[i], kStreamWarps);
        wloaded[i] = -1;
      }
    }
    for (int i = 0; i < kShrinkPartBufs; ++i) {
      mbar_init(&pfull[i], kStreamWarps);
      mbar_init(&pempty[i], 1);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  // slot table staged, barriers initialised, active slots counted
  const int nact = __syncthreads_count(active_mine >= 1) + __syncthreads_count(active_mine >= 2);
  int64_t begin, end;  // this CTA's share, the same in every warp
  // (the fused kernel too: 20-40 tokens measured best for it, 0-10 and 60 slower)
  stream_share(tab, nact, blockIdx.x, gridDim.x, kShrinkSlotCost, lane, begin, end);
  if (begin >= end) return;  // uniform across the CTA
  const uint32_t stage0 = smem_u32(smem);
  const uint32_t row_bytes = (uint32_t)K * 2;
  const uint32_t slot_bytes = (uint32_t)K * (kStreamRank * 2);  // A[slot]: K rows of 32 bytes
  RingSeq it;  // the share's token groups (the producer's and every consumer's own cursor)
  it.init(tab, begin, end, false, false);
  RingItem q;
  bool ok = true;

  if (warp >= kStreamWarps) {
    // ------------------------------------------------ producer warpgroup
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kShrinkProducerRegs));
    if (warp == kStreamWarps) {
      stream_stage_tokens_warp(args.seg.token_index, begin, end, tok_s, lane);
      __syncwarp();
      // the consumers request their weights only now: their 128 KB of loads
      // would otherwise queue ahead of these few bytes
      named_barrier_arrive(kShrinkIdsReady, kStreamThreads + 32);
      const uint64_t pol = l2_evict_first_policy();
      const uint32_t n_row = kFused ? (uint32_t)eargs.N * 2 : 0u;  // one LoRA-B rank row
      int pf_slot = -1;  // slot of the previous group (its rows are in L2 or on their way)
      int ii = 0;
      for (; ok && it.next(tab, begin, q); ++ii) {
        const int s = ii % nst;
        // stage s is free once the 16 consumers released item ii - nst
        if (ii >= nst && !mbar_wait_warp(&empty[s], (uint32_t)(ii / nst - 1) & 1u, abort_flag)) {
          ok = false;
          break;
        }
        if (lane == 0) {
          loaded[s] = ii;
          mbar_arrive_expect_tx(&full[s], (uint32_t)q.cnt * row_bytes);
          if (pf_slot >= 0 && q.slot != pf_slot)  // the consumers load the first slot themselves
            prefetch_l2_bulk(args.a + (int64_t)q.slot * slot_bytes, slot_bytes);
          if (kFused && q.slot != pf_slot)  // the slot's LoRA-B rows, for the expand phase
            prefetch_l2_bulk(eargs.b + (int64_t)q.slot * kStreamRank * n_row,
                             (tab.rk[q.slot] > 8 ? 16u : 8u) * n_row);
        }
        pf_slot = q.slot;
        __syncwarp();
        if (lane < q.cnt)
          bulk_load(stage0 + s * plan.stage_bytes + lane * plan.pitch,
                    args.x + (int64_t)tok_s[q.start + lane] * row_bytes, row_bytes, &full[s], pol);
      }
      if constexpr (kFused) {
        // Weight stage w overwrites the ring stages under it: before its first
        // copy, wait until the consumers have released each of those for the
        // last time (ring stages under neither weight stage, where the tmp rows
        // go, are written only after the consumers' barrier).  The first
        // weight stages so land while the shrink's last groups are consumed.
        int ring_free = 0;  // ring stages [0, ring_free) released for good
        auto free_ring_below = [&](uint32_t bytes) -> bool {
          const int need = min(ii, (int)((bytes + plan.stage_bytes - 1) / plan.stage_bytes));
          for (; ring_free < need; ++ring_free) {
            const int last = ring_free + nst * ((ii - 1 - ring_free) / nst);
            if (!mbar_wait_warp(&empty[ring_free], (uint32_t)(last / nst) & 1u, abort_flag)) return false;
          }
          return true;
        };
        RingSeq wseq;  // the share's weight stages (slots of rank <= 8: only rank rows 0-7)
        wseq.init(tab, begin, end, true, true);
        for (int wi = 0; ok && wseq.next_of(tab, begin, q, true); ++wi) {
          const int w = wi & 1;
          if (wi >= 2 && !mbar_wait_warp(&wempty[w], (uint32_t)(wi / 2 - 1) & 1u, abort_flag)) break;
          if (wi < 2 && !free_ring_below((uint32_t)(w + 1) * fp.w_stage_bytes)) break;
          if (lane == 0) {
            wloaded[w] = wi;
            mbar_arrive_expect_tx(&wfull[w], kStreamGroup * n_row);
          }
          __syncwarp();
          if (lane < kStreamGroup)
            bulk_load(stage0 + w * fp.w_stage_bytes + lane * fp.w_pitch,
                      eargs.b + (((int64_t)q.slot * 2 + q.part) * kStreamGroup + lane) * n_row, n_row, &wfull[w],
                      pol);
        }
      }
    }
  } else {
    // ------------------------------------------------ consumers
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kShrinkConsumerRegs));
    const int g = lane >> 2;  // fragment row group
    const int t = lane & 3;   // lane within the quad
    const int ks = K >> 8;    // k16 steps of this warp's K slice (K / 16 rows)
    const int kw0 = warp * (K >> 4);
    uint32_t a[16][4];  // A^T fragments of the warp's K slice (mma rows g, g + 8; ranks permuted)
    // issues the loads of the slot's fragments in row layout; to_mma_layout() finishes them
    auto load_a = [&](int slot) {
      const uint8_t* src = args.a + (int64_t)slot * slot_bytes + (int64_t)(kw0 + g) * 32 + 8 * t;
#pragma unroll
      for (int j = 0; j < 16; ++j)
        if (j < ks) {
          const uint2 lo = ld_nc_v2(src + j * 16 * 32);
          const uint2 hi = ld_nc_v2(src + j * 16 * 32 + 8 * 32);
          a[j][0] = lo.x;
          a[j][1] = lo.y;
          a[j][2] = hi.x;
          a[j][3] = hi.y;
        }
    };
    auto to_mma_layout = [&]() {
#pragma unroll
      for (int j = 0; j < 16; ++j)
        if (j < ks) {
#pragma unroll
          for (int m = 0; m < 4; ++m) a[j][m] = movmatrix_t(a[j][m]);
        }
    };
    int cur_slot = -1;     // slot whose fragments are in a[] (or on their way)
    bool convert = false;  // a[] holds raw loads still to be transposed
    named_barrier(kShrinkIdsReady, kStreamThreads + 32);  // the producer has its token ids
    {
      RingSeq first = it;
      if (first.next(tab, begin, q)) {  // requested while the first token rows are on their way
        load_a(q.slot);
        cur_slot = q.slot;
        convert = true;
      }
    }
    // ldmatrix row of this lane in a token stage: token row lane & 7, k offset kw0 + 8 (lane >> 3)
    const uint32_t ld_off = (uint32_t)(lane & 7) * plan.pitch + (uint32_t)(kw0 + 8 * (lane >> 3)) * 2;
    uint16_t* tmp = reinterpret_cast<uint16_t*>(args.tmp);
    uint16_t* tile = reinterpret_cast<uint16_t*>(smem + plan.rg_off) + warp * kStreamGroup * kStreamRank;
    int32_t* pmeta = reinterpret_cast<int32_t*>(smem + plan.rg_off + kShrinkTmpTileBytes);  // [3][slot, cnt, start]
    const int rank_lo = shrink_rank_of_row(g), rank_hi = shrink_rank_of_row(g + 8);
    // Adds the 16 partials of group gi (warp order), rounds and writes its tmp
    // rows.  The token ids it reads were staged before stage 0 was armed.
    auto reduce = [&](int gi) -> bool {
      const int pb = gi % kShrinkPartBufs;
      if (!mbar_wait_warp(&pfull[pb], (uint32_t)(gi / kShrinkPartBufs) & 1u, abort_flag)) return false;
      const int g_slot = pmeta[3 * pb], g_cnt = pmeta[3 * pb + 1], g_start = pmeta[3 * pb + 2];
      const float* pp = part + (size_t)pb * (kShrinkPartBytes / 4);
      float v[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int w = 0; w < kStreamWarps; ++w) {
        const float4 u = *reinterpret_cast<const float4*>(pp + (w * 32 + lane) * 4);
        v[0] += u.x;
        v[1] += u.y;
        v[2] += u.z;
        v[3] += u.w;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&pempty[pb]);
      // rounded values -> the warp's tile [token][rank]; then lane l writes 16 bytes
      // (ranks 8 (l & 1) ..) of token l >> 1 with one vector store
      const int n_eff = min(tab.rk[g_slot] * args.stack_num, args.R);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        tile[(2 * t + h) * kStreamRank + rank_lo] = E::from_f(rank_lo < n_eff ? v[h] : 0.f);
        tile[(2 * t + h) * kStreamRank + rank_hi] = E::from_f(rank_hi < n_eff ? v[2 + h] : 0.f);
      }
      __syncwarp();
      if (lane < 2 * g_cnt) {
        const int64_t row = (int64_t)tok_s[g_start + (lane >> 1)] * args.R;
        *reinterpret_cast<uint4*>(tmp + row + 8 * (lane & 1)) = reinterpret_cast<const uint4*>(tile)[lane];
      }
      __syncwarp();
      return true;
    };

    int ii = 0;
    RingItem cq;
    while (it.next(tab, begin, cq)) {
      const int s = ii % nst;
      if (!mbar_wait_warp(&full[s], (uint32_t)(ii / nst) & 1u, abort_flag)) {
        ok = false;
        break;
      }
      if (convert) {
        to_mma_layout();
        convert = false;
      }
      // D^T (mma rows g / g + 8 x token 2t, 2t + 1); stage rows >= cnt hold stale
      // data that only reaches the discarded token columns.  Two accumulators
      // (even / odd k16 steps) halve the dependent mma chain.
      float acc[4] = {0.f, 0.f, 0.f, 0.f}, acc2[4] = {0.f, 0.f, 0.f, 0.f};
      const uint32_t base = stage0 + s * plan.stage_bytes + ld_off;
#pragma unroll
      for (int j = 0; j < 16; j += 2)
        if (j < ks) {
          uint32_t b[4];
          ldsm_x4(base + 32 * j, b);  // k16 steps j and j + 1 of 8 token rows
          mma_16816<BF16>(acc, a[j], b[0], b[1]);
          mma_16816<BF16>(acc2, a[j + 1], b[2], b[3]);
        }
      // the stage's rows have been read (the mma consumed them): release it
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
      // the next group of another slot: its weights are requested now, to land
      // while this group is published and reduced
      {
        RingSeq peek = it;
        RingItem nx;
        if (peek.next(tab, begin, nx) && nx.slot != cur_slot) {
          load_a(nx.slot);
          cur_slot = nx.slot;
          convert = true;
        }
      }
      const int ti = ii++;
      // group ti - 2's reduction falls to warp (ti - 2) mod 16
      const int rg = ti - kShrinkReduceLag;
      if (rg >= 0 && (rg & (kStreamWarps - 1)) == warp && !reduce(rg)) {
        ok = false;
        break;
      }
      // this group's partial -> buffer ti mod 3, once the group 3 earlier has been read
      const int pb = ti % kShrinkPartBufs;
      if (ti >= kShrinkPartBufs &&
          !mbar_wait_warp(&pempty[pb], (uint32_t)(ti / kShrinkPartBufs - 1) & 1u, abort_flag)) {
        ok = false;
        break;
      }
      float* pp = part + (size_t)pb * (kShrinkPartBytes / 4);
      *reinterpret_cast<float4*>(pp + (warp * 32 + lane) * 4) =
          make_float4(acc[0] + acc2[0], acc[1] + acc2[1], acc[2] + acc2[2], acc[3] + acc2[3]);
      if (warp == 0 && lane == 0) {  // the group this buffer now holds, for its reducer
        pmeta[3 * pb] = cq.slot;
        pmeta[3 * pb + 1] = cq.cnt;
        pmeta[3 * pb + 2] = cq.start;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&pfull[pb]);
    }
    // the reductions of the last groups
#pragma unroll
    for (int k = 0; k < kShrinkReduceLag; ++k) {
      const int rg = ii - kShrinkReduceLag + k;
      if (ok && rg >= 0 && (rg & (kStreamWarps - 1)) == warp) ok = reduce(rg);
    }
    if constexpr (kFused) fused_expand_phase<BF16>(eargs, fp, tab, tok_s, begin, end, stage0, abort_flag, wfull,
                                                   wempty, smem, warp, lane);
  }
  __syncthreads();  // every warp is out of its loop
  if (threadIdx.x == 0) {  // the last copy into each stage has landed (unless the roles gave up early)
    for (int s = 0; s < nst; ++s)
      if (loaded[s] >= 0) mbar_drain(&full[s], (uint32_t)(loaded[s] / nst) & 1u);
    if constexpr (kFused)
      for (int w = 0; w < 2; ++w)
        if (wloaded[w] >= 0) mbar_drain(&wfull[w], (uint32_t)(wloaded[w] / 2) & 1u);
  }
}

// ============================================================== expand
// y[t, :] += round(scale * tmp[t, :] @ B[slot(t)]) in place (rank 16), with
// the reference's rounding order; tokens of rank-0 slots and padding are not
// touched.  N % 512 == 0, N <= 4096.
//
// Weight stages (B[slot] rank rows 8p .. 8p + 7 at the stage's row pitch;
// every warp takes the fragments of its columns from both; a slot of rank
// <= 8 has only stage 0, its rows 8..15 entering the mma as zeros) go through
// a ring of two, refilled from their own cursor; the tmp rows of the whole
// share are gathered into shared memory once.
template <bool BF16>
__global__ void __launch_bounds__(kStreamThreads, 1)
    sgmv_expand_stream_kernel(const ExpandArgs args, const StreamPlan plan) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align128(smem_raw);
  const int N = args.N;
  StreamRing wring;
  wring.carve(smem + plan.bar_off, kStreamWeightParts);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + plan.bar_off + kStreamWeightParts * 16);
  int32_t* tok_s = reinterpret_cast<int32_t*>(smem + plan.tok_off);
  int32_t* tab_mem = reinterpret_cast<int32_t*>(smem + plan.tab_off);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const SlotTab tab = stage_slot_tab(args.seg, args.ranks, args.scales, tab_mem);
  if (threadIdx.x == 0) {
    wring.init();
    *abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();  // slot table staged, barriers initialised
  // equal token shares: the weight ring prefetches a slot change, so it adds
  // little to a share's time (charging slot runs as the shrink does measured
  // slower)
  const int64_t total = tab.ss[tab.ns];
  const int64_t begin = total * blockIdx.x / gridDim.x;
  const int64_t end = total * (blockIdx.x + 1) / gridDim.x;
  if (begin >= end) return;  // uniform across the CTA

  const uint32_t stage0 = smem_u32(smem);
  const uint32_t row_bytes = (uint32_t)N * 2;
  const uint64_t pol = l2_evict_first_policy();
  // weight item wi -> weight stage wi % 2
  auto issue_w = [&](int wi, const RingItem& q) {
    ring_issue_weights(wring, wi, args.b + ((int64_t)q.slot * 2 + q.part) * 8 * row_bytes,
                       stage0 + (wi % kStreamWeightParts) * plan.stage_bytes, plan.pitch, row_bytes, pol, lane);
  };
  RingSeq lcw;  // load cursor of the weight stages, 2 ahead
  lcw.init(tab, begin, end, true);
  RingItem q;
  for (int wi = 0; wi < kStreamWeightParts && lcw.next_of(tab, begin, q, true); ++wi)
    if (warp == 0) issue_w(wi, q);
  stream_stage_tokens(args.seg.token_index, begin, end, tok_s);
  __syncthreads();
  // tmp is the previous kernel's output: read only once that grid has completed;
  // every thread gathers 16-byte halves of the share's tmp rows
  griddep_wait();
  const int share = (int)(end - begin);
  for (int i = threadIdx.x; i < 2 * share; i += kStreamThreads)
    cp_async16_cg(stage0 + plan.aux_off + i * 16,
                  args.tmp + (int64_t)tok_s[i >> 1] * kExpandTmpRowBytes + (i & 1) * 16);
  asm volatile("cp.async.commit_group;" ::: "memory");
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  __syncthreads();

  const int g = lane >> 2;  // fragment row group: token g of the group
  const int t = lane & 3;   // lane within the quad
  const int ncw = N >> 4;   // columns of this warp
  const int nt = ncw >> 3;  // n8 tiles of this warp: a multiple of 4, <= 32
  const int c0w = warp * ncw;
  uint32_t b[32][2];  // B fragments of the warp's columns: rank rows 2t.. (+8), column 8 i + g
  // ldmatrix.trans row of this lane in a weight stage: rank row lane & 7, columns c0w + 8 (4 q + (lane >> 3))
  const uint32_t w_off = (uint32_t)(lane & 7) * plan.pitch + (uint32_t)(c0w + 8 * (lane >> 3)) * 2;
  // regroup tile of this warp (8 rows x 64 bytes, 16-byte chunk j of row r at j ^ ((r >> 1) & 3)):
  // stmatrix rows lane & 7 of matrix (tile) lane >> 3; read back row g, columns 8t .. 8t + 7
  const uint32_t rg_base = stage0 + plan.rg_off + warp * kStreamGroup * 64;
  const uint32_t rg_st = rg_base + (lane & 7) * 64 + 16 * ((lane >> 3) ^ (((lane & 7) >> 1) & 3));
  const uint32_t rg_ld = rg_base + g * 64 + 16 * (t ^ ((g >> 1) & 3));
  float scale = 0.f;
  int kr = 0;
  RingSeq it;
  it.init(tab, begin, end, true);
  int wi = 0;
  RingItem cq;
  while (it.next(tab, begin, cq)) {
    if (cq.part >= 0) {  // weight stage: rank rows 8 part .. of this warp's columns
      const int s = wi % kStreamWeightParts;
      if (!mbar_wait_warp(&wring.full[s], (uint32_t)(wi / kStreamWeightParts) & 1u, abort_flag)) break;
      if (cq.part == 0) {
        scale = tab.sc[cq.slot];
        kr = min(tab.rk[cq.slot], args.R);
      }
      const uint32_t sbase = stage0 + s * plan.stage_bytes;
      const bool one_stage = kr <= 8;  // rank rows 8..15 are not loaded and enter as zeros
#pragma unroll
      for (int i = 0; i < 32; i += 4)
        if (i < nt) {
          uint32_t r[4];
          ldsm_x4_t(sbase + w_off + 16 * i, r);  // tiles i .. i + 3 (8 columns, 16 bytes each)
#pragma unroll
          for (int m = 0; m < 4; ++m) {  // register indices must be compile-time
            if (cq.part == 0) {
              b[i + m][0] = r[m];
              if (one_stage) b[i + m][1] = 0u;
            } else {
              b[i + m][1] = r[m];
            }
          }
        }
      const bool last = wring.release(s, lane);
      RingItem nq;
      if (lcw.next_of(tab, begin, nq, true) && last) issue_w(wi + kStreamWeightParts, nq);
      ++wi;
      continue;
    }
    // token group: A fragments from the tmp row of token g (mma rows 8..15 are
    // zero), columns >= kr as zero
    uint32_t fa[4] = {0u, 0u, 0u, 0u};
    const bool vrow = g < cq.cnt;
    int64_t tok = 0;
    if (vrow) {
      const uint32_t* trow =
          reinterpret_cast<const uint32_t*>(smem + plan.aux_off + (cq.start + g) * kExpandTmpRowBytes);
      auto ld2 = [&](int k) -> uint32_t {
        if (k >= kr) return 0u;
        const uint32_t w = trow[k >> 1];
        return k + 1 < kr ? w : (w & 0xFFFFu);
      };
      fa[0] = ld2(2 * t);
      fa[2] = ld2(2 * t + 8);
      tok = tok_s[cq.start + g];
    }
    uint8_t* yrow = args.y + tok * row_bytes + (c0w + 8 * t) * 2;
#pragma unroll
    for (int i = 0; i < 32; i += 4)
      if (i < nt) {  // 32 columns: tiles i .. i + 3
        uint32_t d[4];
#pragma unroll
        for (int m = 0; m < 4; ++m) {
          float acc[4] = {0.f, 0.f, 0.f, 0.f};
          mma_16816<BF16>(acc, fa, b[i + m][0], b[i + m][1]);
          d[m] = pack2<BF16>(scale * acc[0], scale * acc[1]);  // row g, columns 8 (i + m) + 2t, + 1
        }
        stsm_x4(rg_st, d);
        __syncwarp();
        lds_v4(rg_ld, d);  // row g, columns 8 i + 8t .. + 7 of the warp's range
        __syncwarp();
        if (vrow) red_add_v8<BF16>(yrow + 16 * i, d);
      }
  }
  __syncthreads();  // every warp is out of its loop
  if (threadIdx.x == 0) wring.drain();
}

}  // namespace plora
