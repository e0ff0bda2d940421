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
//    lane in mma fragment layout.  The weights arrive as two "weight stages"
//    (LoRA-A halves of K/2 rows; LoRA-B rank rows 0-7 and 8-15) by bulk
//    copies, prefetched like any other stage, and the warps move their slices
//    into registers with ldmatrix.trans.
//  * shrink: token rows travel by one non-multicast `cp.async.bulk` per row
//    (K * 2 bytes) into a ring of shared-memory stages of 8 rows, at a
//    (K * 2 + 16)-byte pitch so that ldmatrix over eight rows hits eight bank
//    groups.  Warp w owns K rows [w K/16, (w + 1) K/16): per stage it
//    multiplies its slice of the 8 rows by its A fragments (mma.sync
//    m16n8k16, D^T = A^T x^T, fp32) and publishes the 16 x 8 partial in
//    shared memory.  Group i's partials are added, in warp order
//    (deterministic), by warp i mod 16 two groups later, which rounds and
//    writes tmp: the reduction is spread over the warps, and by then every
//    warp has long published group i, so the reducer does not wait.
//  * expand: warp w owns N columns [w N/16, (w + 1) N/16).  Per group of 8
//    tokens it computes delta = tmp B for its columns (mma.sync with the tmp
//    rows as A fragments; the share's tmp rows are gathered into shared
//    memory by cp.async once, at the start), rounds scale * delta to
//    the activation type, regroups the fragments so that each lane holds 8
//    consecutive columns of one row (stmatrix into a per-warp tile), and
//    adds them to y with `red.global.add.noftz.v4.{bf16x2,f16x2}`: the L2
//    reads y, adds and rounds to nearest, so y never passes through the SM
//    and nothing waits for it; the result is the reference's (round the
//    scaled delta, then the sum) bit for bit.
// Stages are refilled by the last of the 16 warps to finish with them;
// there is no producer role.  Work split: a CTA per SM takes a contiguous
// share of the slot-ordered token list (its token ids are copied to shared
// memory once, so no global load sits between a stage landing and its
// refill), cut into groups of <= 8 tokens of one slot.  At the start the
// slot table is read first, so that the first weight stages are issued one
// global round trip after launch, while the token ids are still on their way.
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
//   shrink: [nst token/weight stages][3 partial buffers][tmp tiles][group of each buffer][barriers]
//           [token ids][slot table]
//   expand: [2 weight stages][tmp rows of the share][regroup tiles][barriers][token ids][slot table]
// Barrier area: per stage / slot an mbarrier (8 B), a release count and the
// index of the last item loaded (4 B each); then 6 more mbarriers (the
// shrink's partial hand-off) and the abort flag.
struct StreamPlan {
  int nst;               // shrink: ring stages; expand: weight stages
  uint32_t pitch;        // token / weight row pitch in a stage
  uint32_t stage_bytes;  // 8 rows
  uint32_t aux_off;      // shrink: partial buffers; expand: the share's tmp rows
  uint32_t rg_off;       // regroup tiles (shrink: tmp rows of a group; expand: delta columns)
  uint32_t bar_off, tok_off, tab_off;
  uint32_t smem_bytes;   // dynamic shared memory to request (includes 128 B of alignment slack)
};

__host__ __device__ inline uint32_t stream_bar_bytes(int slots) { return (uint32_t)slots * 16 + 6 * 8 + 16; }

__host__ __device__ inline StreamPlan shrink_stream_plan(int64_t K, int64_t num_slots) {
  StreamPlan p;
  p.pitch = (uint32_t)(K * 2 + 16);
  p.stage_bytes = p.pitch * kStreamGroup;
  const int64_t tab = slot_tab_bytes(num_slots);
  const int64_t fixed =
      128 + kShrinkPartBufs * kShrinkPartBytes + kShrinkTmpTileBytes + kShrinkMetaBytes + stream_bar_bytes(0) +
      kStreamMaxShare * 4 + tab;
  int64_t nst = (kStreamSmemLimit - fixed) / ((int64_t)p.stage_bytes + 16);
  if (nst > kStreamMaxStages) nst = kStreamMaxStages;
  p.nst = (int)nst;
  p.aux_off = (uint32_t)(nst * p.stage_bytes);
  p.rg_off = p.aux_off + kShrinkPartBufs * kShrinkPartBytes;
  p.bar_off = p.rg_off + kShrinkTmpTileBytes + kShrinkMetaBytes;
  p.tok_off = p.bar_off + stream_bar_bytes(p.nst);
  p.tab_off = p.tok_off + kStreamMaxShare * 4;
  p.smem_bytes = (uint32_t)(128 + p.tab_off + tab);
  return p;
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

// Bounded wait that ignores the abort flag: used to let copies already issued
// land before the CTA exits.  Its limit is the fixed 1 s, not the settable
// wait limit: a copy in flight takes microseconds, and a shortened limit must
// not let a CTA exit while one still writes its shared memory.  Returns false
// on expiry (status raised).
__device__ __forceinline__ bool mbar_drain(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  for (;;) {
    if (mbar_try_wait_parked(bar, parity)) return true;
    if (global_timer_ns() - t0 > kWaitLimitNs) {
      raise_status(PLORA_DEV_WAIT_TIMEOUT);
      return false;
    }
  }
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
// CTA's share of the slot-ordered token list, the slot's two weight stages,
// then its groups of <= 8 tokens (runs of rank-0 slots are skipped).
// Positions are relative to the share's start `base`.
struct RingItem {
  int part;  // weight stage 0 / 1, or -1 for a token group
  int slot, cnt, start;
};

struct RingSeq {
  int p, end, slot, wslot, wpart;  // wslot: slot whose weight stages were last emitted
  bool low_half_only;              // slots of rank <= 8 need only weight stage 0 (expand)
  __device__ void init(const SlotTab& t, int64_t b, int64_t e, bool rank8_one_stage = false) {
    p = 0;
    end = (int)(e - b);
    slot = (b < e) ? slot_of_position(t.ss, t.ns, b) : 0;
    wslot = -1;
    wpart = 0;
    low_half_only = rank8_one_stage;
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
      if (slot != wslot) {
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

// ============================================================== shrink
// tmp[t, :] = x[t, :] @ A[slot(t)] (rank 16) for the active tokens of the
// table; columns >= min(rank * stack_num, 16) of an active token are written
// as 0, inactive tokens are not written.  K % 512 == 0, K <= 4096.
//
// Weight stage p holds A[slot] rows [p K/2, (p + 1) K/2) (32 bytes each,
// contiguous); warps 8p .. 8p + 7 take their K slices from it.
template <bool BF16>
__global__ void __launch_bounds__(kStreamThreads, 1)
    sgmv_shrink_stream_kernel(const ShrinkArgs args, const StreamPlan plan) {
  using E = Elem<BF16>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align128(smem_raw);
  const int nst = plan.nst;
  const int K = args.K;
  float* part = reinterpret_cast<float*>(smem + plan.aux_off);
  StreamRing ring;
  ring.carve(smem + plan.bar_off, nst);
  uint64_t* pfull = reinterpret_cast<uint64_t*>(ring.loaded + nst);  // [3] all 16 partials of the group written
  uint64_t* pempty = pfull + kShrinkPartBufs;                          // [3] the group's partials have been read
  volatile int* abort_flag = reinterpret_cast<volatile int*>(pempty + kShrinkPartBufs);
  int32_t* tok_s = reinterpret_cast<int32_t*>(smem + plan.tok_off);
  int32_t* tab_mem = reinterpret_cast<int32_t*>(smem + plan.tab_off);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  griddep_wait();    // inputs (segment table, x) come from earlier kernels
  griddep_launch();  // the expand may start on SMs this grid releases
  const SlotTab tab = stage_slot_tab(args.seg, args.ranks, nullptr, tab_mem);
  if (threadIdx.x == 0) {
    ring.init();
    for (int i = 0; i < kShrinkPartBufs; ++i) {
      mbar_init(&pfull[i], kStreamWarps);
      mbar_init(&pempty[i], 1);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();  // slot table staged, barriers initialised
  const int64_t total = tab.ss[tab.ns];
  const int64_t begin = total * blockIdx.x / gridDim.x;
  const int64_t end = total * (blockIdx.x + 1) / gridDim.x;
  if (begin >= end) return;  // uniform across the CTA
  const uint32_t stage0 = smem_u32(smem);
  const uint32_t row_bytes = (uint32_t)K * 2;
  const uint64_t pol = l2_evict_first_policy();
  // item ii: a weight stage (8 contiguous K*2-byte pieces of A[slot]) or 8 token rows
  auto issue = [&](int ii, const RingItem& q) {
    const int s = ii % nst;
    const uint32_t dst = stage0 + s * plan.stage_bytes;
    if (q.part >= 0) {
      ring_issue_weights(ring, ii, args.a + ((int64_t)q.slot * 2 + q.part) * 8 * row_bytes, dst, row_bytes, row_bytes,
                         pol, lane);
      return;
    }
    if (lane == 0) ring_arm(ring, s, ii, (uint32_t)q.cnt * row_bytes);
    __syncwarp();
    if (lane < q.cnt)
      bulk_load(dst + lane * plan.pitch, args.x + (int64_t)tok_s[q.start + lane] * row_bytes, row_bytes,
                &ring.full[s], pol);
  };

  RingSeq lc;  // load cursor: nst items ahead of consumption; warp 0 issues the first nst
  lc.init(tab, begin, end);
  RingItem q;
  {
    // weight stages first (they need only the table), token stages once the ids are staged
    RingSeq pre = lc;
    for (int ii = 0; ii < nst && pre.next(tab, begin, q); ++ii)
      if (warp == 0 && q.part >= 0) issue(ii, q);
    stream_stage_tokens(args.seg.token_index, begin, end, tok_s);
    __syncthreads();
    for (int ii = 0; ii < nst && lc.next(tab, begin, q); ++ii)
      if (warp == 0 && q.part < 0) issue(ii, q);
  }

  const int g = lane >> 2;  // fragment row group
  const int t = lane & 3;   // lane within the quad
  const int ks = K >> 8;    // k16 steps of this warp's K slice (K / 16 rows)
  const int kw0 = warp * (K >> 4);
  const int my_part = warp / (kStreamWarps / kStreamWeightParts);
  uint32_t a[16][4];  // A^T fragments of the warp's K slice (rank rows g, g + 8)
  // ldmatrix row of this lane in a token stage: token row lane & 7, k offset kw0 + 8 (lane >> 3)
  const uint32_t ld_off = (uint32_t)(lane & 7) * plan.pitch + (uint32_t)(kw0 + 8 * (lane >> 3)) * 2;
  // ldmatrix.trans row of this lane in its weight stage: k = 16 j + 8 (m >> 1) + (lane & 7)
  // of the warp's slice, rank half m & 1, for matrix m = lane >> 3
  const uint32_t w_off = (uint32_t)(kw0 - my_part * (K >> 1) + 8 * (lane >> 4) + (lane & 7)) * 32 +
                         16 * ((lane >> 3) & 1);
  uint16_t* tmp = reinterpret_cast<uint16_t*>(args.tmp);
  uint16_t* tile = reinterpret_cast<uint16_t*>(smem + plan.rg_off) + warp * kStreamGroup * kStreamRank;
  int32_t* pmeta = reinterpret_cast<int32_t*>(smem + plan.rg_off + kShrinkTmpTileBytes);  // [3][slot, cnt, start]
  // Adds the 16 partials of group gi (warp order), rounds and writes its tmp rows.
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
      tile[(2 * t + h) * kStreamRank + g] = E::from_f(g < n_eff ? v[h] : 0.f);
      tile[(2 * t + h) * kStreamRank + g + 8] = E::from_f(g + 8 < n_eff ? v[2 + h] : 0.f);
    }
    __syncwarp();
    if (lane < 2 * g_cnt) {
      const int64_t row = (int64_t)tok_s[g_start + (lane >> 1)] * args.R;
      *reinterpret_cast<uint4*>(tmp + row + 8 * (lane & 1)) = reinterpret_cast<const uint4*>(tile)[lane];
    }
    __syncwarp();
    return true;
  };

  RingSeq it;
  it.init(tab, begin, end);
  int ii = 0, ti = 0;
  RingItem cq;
  bool ok = true;
  while (it.next(tab, begin, cq)) {
    const int s = ii % nst;
    if (!mbar_wait_warp(&ring.full[s], (uint32_t)(ii / nst) & 1u, abort_flag)) {
      ok = false;
      break;
    }
    const uint32_t sbase = stage0 + s * plan.stage_bytes;
    // two accumulators (even / odd k16 steps) halve the dependent mma chain
    float acc[4] = {0.f, 0.f, 0.f, 0.f}, acc2[4] = {0.f, 0.f, 0.f, 0.f};
    if (cq.part >= 0) {  // weight stage: the warps of this half take their A fragments
      if (cq.part == my_part) {
#pragma unroll
        for (int j = 0; j < 16; ++j)
          if (j < ks) ldsm_x4_t(sbase + w_off + 16 * 32 * j, a[j]);
      }
    } else {
      // D^T (rank g / g + 8 x token 2t, 2t + 1); stage rows >= cnt hold stale
      // data that only reaches the discarded token columns
      const uint32_t base = sbase + ld_off;
#pragma unroll
      for (int j = 0; j < 16; j += 2)
        if (j < ks) {
          uint32_t b[4];
          ldsm_x4(base + 32 * j, b);  // k16 steps j and j + 1 of 8 token rows
          mma_16816<BF16>(acc, a[j], b[0], b[1]);
          mma_16816<BF16>(acc2, a[j + 1], b[2], b[3]);
        }
    }
    // the 16th warp out of the stage refills it with item ii + nst
    const bool refill = ring.release(s, lane);
    RingItem nq;
    if (lc.next(tab, begin, nq) && refill) issue(ii + nst, nq);
    ++ii;
    if (cq.part >= 0) continue;

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
    ++ti;
  }
  // the reductions of the last groups
#pragma unroll
  for (int k = 0; k < kShrinkReduceLag; ++k) {
    const int rg = ti - kShrinkReduceLag + k;
    if (ok && rg >= 0 && (rg & (kStreamWarps - 1)) == warp) ok = reduce(rg);
  }
  __syncthreads();  // every warp is out of its loop
  if (threadIdx.x == 0) ring.drain();
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
