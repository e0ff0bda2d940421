// SGMV shrink and expand on the 5th-generation tensor cores (tcgen05 + TMEM),
// bf16/fp16 operands with fp32 accumulation.
//
// Both kernels walk the device segment table (slot_start / token_index):
// active tokens are grouped by slot, so one slot's LoRA weights are staged
// in shared memory once per tile of up to 128 tokens and a single elected
// thread issues tcgen05.mma into a TMEM accumulator.  All bulk data moves on
// the TMA engine into this CTA's own shared memory: the scattered token rows
// of x by tile::gather4 (four rows per instruction, 128-byte swizzled straight
// into the UMMA operand layout), the per-slot weight tiles by tiled TMA, and
// the rows of y by 1-D bulk copies in and out.  Work is split evenly over a
// persistent grid: shrink by tokens, expand by tokens x 128-column tiles.
//
// Reference semantics: src/polylora/sgmv.py:63-138 (_sgmv_lora_a_kernel) and
// sgmv.py:178-275 (_sgmv_lora_b_kernel).
#pragma once

#include "common.cuh"

namespace plora {

constexpr int kTileM = 128;        // tokens per MMA tile (TMEM lanes)
constexpr int kShrinkKC = 64;      // K elements per shrink stage (one 128-byte row)
constexpr int kExpandNT = 128;     // output columns per expand unit
constexpr int kShrinkThreads = 704;  // 16 producer warps, A TMA, MMA, 4 epilogue warps
constexpr int kExpandThreads = 768;  // B TMA, MMA, tmp gather, idle, 4 TMEM readers, 16 y streams

struct SegTable {
  const int32_t* slot_start;   // (num_slots + 1)
  const int32_t* token_index;  // (>= slot_start[num_slots])
  int32_t num_slots;
};

struct ShrinkArgs {
  const uint8_t* x;   // (tokens, K)
  const uint8_t* a;   // (NS, K, R)   (SIMT path; the TC path reads it by TMA)
  uint8_t* tmp;       // (tokens, R)
  const int32_t* ranks;
  SegTable seg;
  int32_t K, R, stack_num;
};

struct ExpandArgs {
  const uint8_t* tmp;  // (tokens, R)
  const uint8_t* b;    // (NS, R, N)  (SIMT path)
  uint8_t* y;          // (tokens, N)
  const int32_t* ranks;
  const float* scales;
  SegTable seg;
  int32_t R, N;
};

// Per-slot metadata staged in shared memory once per CTA (slot_start, ranks
// and, for the expand, scales), so the schedule never waits on global loads.
constexpr int kTcMaxSlots = 1024;  // slot-count limit of the tensor-core kernels

struct SlotTab {
  const int32_t* ss;  // (num_slots + 1) slot_start
  const int32_t* rk;  // (num_slots) ranks of this module
  const float* sc;    // (num_slots) scales (expand only)
  int ns;
};

__device__ __forceinline__ size_t slot_tab_bytes(int ns) { return (size_t)(3 * ns + 1) * 4; }

// Copies the table into `dst` (all threads of the CTA; caller syncs).
__device__ __forceinline__ SlotTab stage_slot_tab(const SegTable& t, const int32_t* ranks,
                                                  const float* scales, int32_t* dst) {
  const int ns = t.num_slots;
  int32_t* ss = dst;
  int32_t* rk = dst + ns + 1;
  float* sc = reinterpret_cast<float*>(dst + 2 * ns + 1);
  for (int i = threadIdx.x; i <= ns; i += blockDim.x) ss[i] = __ldg(t.slot_start + i);
  for (int i = threadIdx.x; i < ns; i += blockDim.x) {
    rk[i] = __ldg(ranks + i);
    sc[i] = scales ? __ldg(scales + i) : 0.f;
  }
  return SlotTab{ss, rk, sc, ns};
}

// Items of the shrink: maximal runs of <= 128 tokens of one slot inside the
// CTA's contiguous share [p, end) of the slot-ordered token list.
struct ShrinkItems {
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
    cnt = (int)min(lim - p, (int64_t)kTileM);
    s = slot;
    start = p;
    p += cnt;
    return true;
  }
};

// Units of the expand: the work space is (token, 128-column tile) pairs laid
// out slot-major, then 128-token item, then column tile, then token.  A CTA
// takes a contiguous share; a unit is one (item, column tile) with the token
// sub-range [t0, t1) of the item that falls inside the share.  The cursor
// advances incrementally; only init() searches.
struct ExpandUnit {
  int slot;
  int64_t item_start;  // first position of the item in token_index
  int cnt;             // tokens in the item
  int tile;            // output column tile
  int t0, t1;          // token sub-range of this unit
};

struct ExpandUnits {
  int64_t w, wend;
  int ntiles;
  int s, item, cnt, tile, t;
  int64_t s0, cnt_s;
  __device__ void init(const SlotTab& tab, int64_t b, int64_t e, int nt) {
    w = b;
    wend = e;
    ntiles = nt;
    if (b >= e) return;
    int lo = 0, hi = tab.ns - 1;  // largest s with ss[s] * nt <= w
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if ((int64_t)tab.ss[mid] * nt <= w)
        lo = mid;
      else
        hi = mid - 1;
    }
    s = lo;
    s0 = tab.ss[s];
    cnt_s = (int64_t)tab.ss[s + 1] - s0;
    const int64_t local = w - s0 * nt;
    item = (int)(local / ((int64_t)kTileM * nt));
    cnt = (int)min((int64_t)kTileM, cnt_s - (int64_t)item * kTileM);
    const int64_t within = local - (int64_t)item * kTileM * nt;
    tile = (int)(within / cnt);
    t = (int)(within % cnt);
  }
  __device__ bool next(const SlotTab& tab, ExpandUnit& u) {
    if (w >= wend) return false;
    u.slot = s;
    u.item_start = s0 + (int64_t)item * kTileM;
    u.cnt = cnt;
    u.tile = tile;
    u.t0 = t;
    const int64_t take = min((int64_t)(cnt - t), wend - w);
    u.t1 = t + (int)take;
    w += take;
    t = u.t1;
    if (w < wend && t == cnt) {  // advance to the next (item, tile)
      t = 0;
      if (++tile == ntiles) {
        tile = 0;
        if ((int64_t)(++item) * kTileM >= cnt_s) {
          item = 0;
          do {
            ++s;
          } while (tab.ss[s + 1] == tab.ss[s]);  // w < wend: a later non-empty slot exists
          s0 = tab.ss[s];
          cnt_s = (int64_t)tab.ss[s + 1] - s0;
        }
        cnt = (int)min((int64_t)kTileM, cnt_s - (int64_t)item * kTileM);
      }
    }
    return true;
  }
};

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~(uintptr_t)1023);
}

// Time-bounded wait that ignores the abort flag (used to drain own work).
__device__ __forceinline__ void mbar_drain(uint64_t* bar, uint32_t parity) {
  const uint64_t t0 = global_timer_ns();
  while (!mbar_try_wait_parked(bar, parity)) {
    if (global_timer_ns() - t0 > kWaitLimitNs) {
      raise_status(PLORA_DEV_WAIT_TIMEOUT);
      return;
    }
  }
}

// ============================================================== shrink
constexpr int kShrinkProducerWarps = 16;
constexpr int kShrinkMaxStages = 32;
constexpr int kShrinkRingBytes = 144 * 1024;  // stage ring budget (x tile + A chunk per stage)
#ifndef PLORA_SHRINK_PREFETCH
#define PLORA_SHRINK_PREFETCH 0
#endif
constexpr int kShrinkPrefetch = PLORA_SHRINK_PREFETCH;  // chunk groups fetched into L2 ahead of the register loads

template <int RP>
struct ShrinkCfg {
  static constexpr int kABytes = kShrinkKC * RP * 2;  // MN-major, swizzle = RP*2 bytes
  static constexpr int kTmemCols = (2 * RP < 32) ? 32 : 2 * RP;
  static constexpr uint32_t kALayout = RP == 16 ? kSwizzle32 : (RP == 32 ? kSwizzle64 : kSwizzle128);
  static constexpr uint32_t kAAtom = 8 * RP * 2;  // 8 K-rows of one swizzle atom
  static constexpr int kBarrierBytes = 1024;
  // ring + tail pad (the UMMA reads 128 rows from any stage) + barriers;
  // + slot table (3 * num_slots + 1 ints), sized at launch
  static constexpr int kSmemBytes = 1024 + kShrinkRingBytes + kTileM * 128 + kBarrierBytes;
};

// tmp[t, :] = x[t, :] @ A[slot(t)] for the active tokens of the table.
//   warps 0-15: producers, one warp per token row: a warp-wide 16-byte load
//           covers four 64-wide K chunks of one row (512 contiguous bytes);
//           the next group of chunks is loaded while the current one is
//           stored into the 128-byte-swizzled K-major stage tiles.
//   warp 16: TMEM owner; lane 0 loads A[slot] (64 x RP) per stage by TMA.
//   warp 17: lane 0 issues 4 UMMAs (128 x RP x 16) per stage.
//   warps 18-21: epilogue — TMEM -> registers -> bf16/fp16 rows of tmp.
// Stage tiles are `rows_pad` rows apart (the CTA's largest item rounded up
// to 8): the UMMA reads 128 rows per stage and ignores the rows past the
// item, so small items do not waste the ring.
template <int RP, bool BF16>
__global__ void __launch_bounds__(kShrinkThreads, 1)
    sgmv_shrink_tc_kernel(const __grid_constant__ CUtensorMap tmap_a, const ShrinkArgs args) {
  using Cfg = ShrinkCfg<RP>;
  using E = Elem<BF16>;
  constexpr int PW = kShrinkProducerWarps;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kShrinkRingBytes + kTileM * 128);
  uint64_t* empty = full + kShrinkMaxStages;
  uint64_t* acc_full = empty + kShrinkMaxStages;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int32_t* tab_mem = reinterpret_cast<int32_t*>(smem + kShrinkRingBytes + kTileM * 128 + Cfg::kBarrierBytes);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t total = __ldg(args.seg.slot_start + args.seg.num_slots);
  const int64_t begin = total * blockIdx.x / gridDim.x;
  const int64_t end = total * (blockIdx.x + 1) / gridDim.x;
  if (begin >= end) return;  // uniform across the CTA

  const SlotTab tab = stage_slot_tab(args.seg, args.ranks, nullptr, tab_mem);
  __syncthreads();
  // ring geometry from the CTA's largest item
  int max_cnt = 1;
  {
    ShrinkItems it;
    it.init(tab, begin, end);
    int s, c;
    int64_t st;
    while (it.next(tab, s, st, c)) max_cnt = max(max_cnt, c);
  }
  const int rows_pad = (max_cnt + 7) & ~7;
  const int stage_bytes = rows_pad * 128 + Cfg::kABytes;  // x tile then A chunk, 1024-aligned
  const int S = min(kShrinkMaxStages, kShrinkRingBytes / stage_bytes);

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], PW + 1);  // producer warps + the A loader's expect_tx
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 4);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == PW) {
    tmem_alloc(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int nkc = (args.K + kShrinkKC - 1) / kShrinkKC;
  const int ngroups = (nkc + 3) >> 2;
  const uint32_t ring = smem_u32(smem);

  ShrinkItems items;
  items.init(tab, begin, end);
  int s, cnt;
  int64_t start;

  if (warp < PW) {
    // ---------------- producers: rows warp + 16 i of each item, four at a time
    const int sub = lane >> 3;  // which of the 4 chunks of a group this lane loads
    const int pc = lane & 7;    // 16-byte piece within the 128-byte chunk
    uint32_t base_ctr = 0;      // stage counter of the item's first chunk
    bool ok = true;
    while (ok && items.next(tab, s, start, cnt)) {
      if (tab.rk[s] <= 0) continue;
      const int nrows = cnt > warp ? (cnt - warp + PW - 1) / PW : 0;  // <= 8
      const int nrb = nrows > 4 ? 2 : 1;  // row blocks; a warp without rows still arrives
      const int tok_mine = lane < nrows ? __ldg(args.seg.token_index + start + warp + PW * lane) : 0;
      const int npairs = ngroups * nrb;  // (chunk group, row block) steps, group-major
      // loads rows 4 rb .. 4 rb + 3 of this warp for chunk group g
      auto load = [&](int p, uint4 (&dst)[4]) {
        const int g = p / nrb, rb = p - g * nrb;
        const int k0 = (4 * g + sub) * kShrinkKC + pc * 8;
        if (kShrinkPrefetch > 0 && rb == 0) {  // lines of group g + kShrinkPrefetch into L2
          const int kp = (4 * (g + kShrinkPrefetch) + sub) * kShrinkKC;
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int tok = __shfl_sync(0xffffffffu, tok_mine, i);
            if (pc == 0 && i < nrows && kp < args.K) prefetch_l2(args.x + ((int64_t)tok * args.K + kp) * 2);
          }
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int i = 4 * rb + j;
          const int tok = __shfl_sync(0xffffffffu, tok_mine, i);
          if (i < nrows && k0 < args.K)
            dst[j] = __ldg(reinterpret_cast<const uint4*>(args.x + ((int64_t)tok * args.K + k0) * 2));
          else
            dst[j] = make_uint4(0u, 0u, 0u, 0u);
        }
      };
      // stores step p into its stages; the first row block waits for the
      // stages to be free, the last one publishes them
      auto store = [&](int p, const uint4 (&src)[4]) -> bool {
        const int g = p / nrb, rb = p - g * nrb;
        if (rb == 0) {
          for (int q = 0; q < 4; ++q) {
            const int kc = 4 * g + q;
            if (kc >= nkc) break;
            const uint32_t ctr = base_ctr + kc;
            if (!mbar_wait_warp(&empty[ctr % S], ((ctr / S) & 1) ^ 1, abort_flag)) return false;
          }
        }
        const int kc = 4 * g + sub;
        const uint32_t st = (base_ctr + kc) % S;
        if (kc < nkc) {
          const uint32_t xs = ring + st * stage_bytes;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int i = 4 * rb + j;
            if (i < nrows) {
              const int r = warp + PW * i;
              const uint32_t dst = xs + r * 128 + ((pc ^ (r & 7)) << 4);
              asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(dst), "r"(src[j].x),
                           "r"(src[j].y), "r"(src[j].z), "r"(src[j].w)
                           : "memory");
            }
          }
        }
        if (rb == nrb - 1) {
          fence_proxy_async_smem();
          __syncwarp();
          if (pc == 0 && kc < nkc) mbar_arrive(&full[st]);  // one arrival per warp per stage
        }
        return true;
      };
      uint4 ra[4], rb_[4];
      load(0, ra);
      for (int p = 0; p < npairs; p += 2) {
        if (p + 1 < npairs) load(p + 1, rb_);
        if (!store(p, ra)) {
          ok = false;
          break;
        }
        if (p + 1 >= npairs) break;
        if (p + 2 < npairs) load(p + 2, ra);
        if (!store(p + 1, rb_)) {
          ok = false;
          break;
        }
      }
      base_ctr += nkc;
    }
  } else if (warp == PW) {
    // ---------------- A chunk loader (TMA)
    if (lane == 0) {
      prefetch_tmap(&tmap_a);
      uint32_t ctr = 0;
      bool ok = true;
      while (ok && items.next(tab, s, start, cnt)) {
        if (tab.rk[s] <= 0) continue;
        for (int kc = 0; kc < nkc; ++kc, ++ctr) {
          const int st = ctr % S;
          if (!mbar_wait(&empty[st], ((ctr / S) & 1) ^ 1, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[st], Cfg::kABytes);
          tma_load_3d(ring + st * stage_bytes + rows_pad * 128, &tmap_a, &full[st], 0,
                      kc * kShrinkKC, s);
        }
      }
    }
  } else if (warp == PW + 1) {
    // ---------------- MMA issue (one thread)
    if (lane == 0) {
      const uint32_t idesc = idesc_f16(BF16, false, true, kTileM, RP);
      uint32_t ctr = 0, item_ctr = 0;
      bool issued = false, ok = true;
      while (ok && items.next(tab, s, start, cnt)) {
        if (tab.rk[s] <= 0) continue;
        const int ab = item_ctr & 1;
        if (!mbar_wait(&acc_empty[ab], ((item_ctr >> 1) & 1) ^ 1, abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + ab * RP;
        for (int kc = 0; kc < nkc; ++kc, ++ctr) {
          const int st = ctr % S;
          if (!mbar_wait(&full[st], (ctr / S) & 1, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t xs = ring + st * stage_bytes;
          const uint32_t as = xs + rows_pad * 128;
#pragma unroll
          for (int kk = 0; kk < kShrinkKC / 16; ++kk) {
            const uint64_t adesc = smem_desc(xs + kk * 32, 16, 1024, kSwizzle128);
            const uint64_t bdesc =
                smem_desc(as + kk * 2 * Cfg::kAAtom, Cfg::kAAtom, Cfg::kAAtom, Cfg::kALayout);
            umma_f16(d_tmem, adesc, bdesc, idesc, (kc | kk) != 0);
          }
          umma_commit(&empty[st]);
          issued = true;
        }
        if (!ok) break;
        umma_commit(&acc_full[ab]);
        ++item_ctr;
      }
      if (issued) {
        umma_commit(drain);
        mbar_drain(drain, 0);
      }
    }
  } else {
    // ---------------- epilogue: TMEM -> registers -> tmp rows
    const int q = warp & 3;  // TMEM lane quarter of this warp
    const int r = q * 32 + lane;
    uint32_t item_ctr = 0;
    while (items.next(tab, s, start, cnt)) {
      const int rank = tab.rk[s];
      if (rank <= 0) continue;
      const int64_t tok = (r < cnt) ? __ldg(args.seg.token_index + start + r) : 0;
      const int ab = item_ctr & 1;
      if (!mbar_wait_warp(&acc_full[ab], (item_ctr >> 1) & 1, abort_flag)) break;
      tc_fence_after();
      uint32_t v[RP / 16][16];
#pragma unroll
      for (int g = 0; g < RP / 16; ++g)
        tmem_ld16(tmem_base + ((uint32_t)(q * 32) << 16) + ab * RP + g * 16, v[g]);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[ab]);
      if (r < cnt) {
        const int n_eff = min(rank * args.stack_num, args.R);
        uint4* dst = reinterpret_cast<uint4*>(args.tmp + tok * args.R * 2);
#pragma unroll
        for (int ch = 0; ch < RP / 8; ++ch) {
          uint32_t w[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int j0 = ch * 8 + 2 * i;
            const float f0 = (j0 < n_eff) ? __uint_as_float(v[j0 >> 4][j0 & 15]) : 0.f;
            const float f1 = (j0 + 1 < n_eff) ? __uint_as_float(v[(j0 + 1) >> 4][(j0 + 1) & 15]) : 0.f;
            w[i] = (uint32_t)E::from_f(f0) | ((uint32_t)E::from_f(f1) << 16);
          }
          dst[ch] = make_uint4(w[0], w[1], w[2], w[3]);
        }
      }
      ++item_ctr;
    }
  }

  __syncthreads();
  if (warp == PW) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::kTmemCols);
  }
}

// ============================================================== expand
constexpr int kExpandStreamWarps = 16;
constexpr int kDeltaRowBytes = kExpandNT * 2 + 16;  // padded smem row: conflict-free both ways
#ifndef PLORA_EXPAND_PREFETCH
#define PLORA_EXPAND_PREFETCH 4
#endif
constexpr int kExpandPrefetch = PLORA_EXPAND_PREFETCH;  // column tiles of the same rows fetched into L2 ahead

template <int RP>
struct ExpandCfg {
  static constexpr int kBoxBytes = RP * 128;  // RP rows x 64 columns, MN-major SW128
  static constexpr int kBStageBytes = 2 * kBoxBytes;
  static constexpr int kBStageStride = (kBStageBytes + 1023) & ~1023;
  static constexpr int kTmpBytes = kTileM * RP * 2;  // K-major, no swizzle
  static constexpr int kDeltaBytes = kTileM * kDeltaRowBytes;
  static constexpr int kBStages = 4;  // LoRA-B tile stages
  static constexpr int kTmemCols = 2 * kExpandNT;
  static constexpr int kBarrierBytes = 512;
  // + slot table (3 * num_slots + 1 ints), sized at launch
  static constexpr int kSmemBytes =
      1024 + kBStages * kBStageStride + 2 * kTmpBytes + 2 * kDeltaBytes + kBarrierBytes;
};

// Register set of one stream warp for one unit: four 16-byte y pieces (rows
// 32 j + 2 w + h, piece c of the 256-byte row segment) and their token rows.
struct YSet {
  uint4 v[4];
  int32_t tok[4];
  int n0;
  uint32_t mask;  // bit j: piece j is active
};

// y[t, :] += round(scale[slot(t)] * tmp[t, :] @ B[slot(t)]) (in place), the
// reference's order: the fp32 product is scaled, rounded to the activation
// type, then added to the base output.
//   warp 0: lane 0 loads the B tile (RP x 128) per unit by TMA.
//   warp 1: TMEM owner; lane 0 issues RP/16 UMMAs (128 x 128 x 16) per unit.
//   warp 2: gathers the item's tmp rows (K-major, no swizzle) with cp.async.
//   warps 4-7: TMEM readers — thread = token row: scaled, rounded delta rows
//           into a double-buffered padded smem tile.
//   warps 8-23: y streams — a half warp per 256-byte row segment, 16-byte
//           loads issued one unit ahead into registers, delta added from
//           smem, 16-byte stores back in place.
template <int RP, bool BF16>
__global__ void __launch_bounds__(kExpandThreads, 1)
    sgmv_expand_tc_kernel(const __grid_constant__ CUtensorMap tmap_b, const ExpandArgs args) {
  using Cfg = ExpandCfg<RP>;
  using E = Elem<BF16>;
  constexpr int S = Cfg::kBStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* bst_base = smem;
  uint8_t* tmp_base = smem + S * Cfg::kBStageStride;
  uint8_t* d_base = tmp_base + 2 * Cfg::kTmpBytes;
  uint64_t* bfull = reinterpret_cast<uint64_t*>(d_base + 2 * Cfg::kDeltaBytes);
  uint64_t* bempty = bfull + S;
  uint64_t* tfull = bempty + S;
  uint64_t* tempty = tfull + 2;
  uint64_t* afull = tempty + 2;
  uint64_t* aempty = afull + 2;
  uint64_t* dfull = aempty + 2;
  uint64_t* dempty = dfull + 2;
  uint64_t* drain = dempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int32_t* tab_mem = reinterpret_cast<int32_t*>(d_base + 2 * Cfg::kDeltaBytes + Cfg::kBarrierBytes);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int ntiles = (args.N + kExpandNT - 1) / kExpandNT;
  const int64_t total = (int64_t)__ldg(args.seg.slot_start + args.seg.num_slots) * ntiles;
  const int64_t begin = total * blockIdx.x / gridDim.x;
  const int64_t end = total * (blockIdx.x + 1) / gridDim.x;
  if (begin >= end) return;

  const SlotTab tab = stage_slot_tab(args.seg, args.ranks, args.scales, tab_mem);
  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&bfull[i], 1);
      mbar_init(&bempty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 32);
      mbar_init(&tempty[i], 1);
      mbar_init(&afull[i], 1);
      mbar_init(&aempty[i], 4);
      mbar_init(&dfull[i], 4);
      mbar_init(&dempty[i], kExpandStreamWarps);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  ExpandUnits units;
  units.init(tab, begin, end, ntiles);
  ExpandUnit u;

  if (warp == 0) {
    // ---------------- B tile loader (TMA)
    if (lane == 0) {
      prefetch_tmap(&tmap_b);
      uint32_t bctr = 0;
      while (units.next(tab, u)) {
        if (tab.rk[u.slot] <= 0) continue;
        const int st = bctr % S;
        if (!mbar_wait(&bempty[st], ((bctr / S) & 1) ^ 1, abort_flag)) break;
        mbar_arrive_expect_tx(&bfull[st], Cfg::kBStageBytes);
        const uint32_t dst = smem_u32(bst_base + st * Cfg::kBStageStride);
        const int n0 = u.tile * kExpandNT;
        tma_load_3d(dst, &tmap_b, &bfull[st], n0, 0, u.slot);
        tma_load_3d(dst + Cfg::kBoxBytes, &tmap_b, &bfull[st], n0 + 64, 0, u.slot);
        ++bctr;
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issue (one thread)
    if (lane == 0) {
      const uint32_t idesc = idesc_f16(BF16, false, true, kTileM, kExpandNT);
      uint32_t bctr = 0, unit_ctr = 0, item_ctr = 0;
      int64_t prev = -1;
      int tb = 0;
      bool issued = false, ok = true;
      while (ok && units.next(tab, u)) {
        if (tab.rk[u.slot] <= 0) continue;
        if (u.item_start != prev) {
          if (prev >= 0) umma_commit(&tempty[tb]);  // previous tile free once its MMAs finish
          prev = u.item_start;
          tb = item_ctr & 1;
          if (!mbar_wait(&tfull[tb], (item_ctr >> 1) & 1, abort_flag)) {
            ok = false;
            break;
          }
          fence_proxy_async_smem();  // cp.async (generic proxy) data -> UMMA operand
          ++item_ctr;
        }
        const int st = bctr % S;
        if (!mbar_wait(&bfull[st], (bctr / S) & 1, abort_flag)) break;
        const int ab = unit_ctr & 1;
        if (!mbar_wait(&aempty[ab], ((unit_ctr >> 1) & 1) ^ 1, abort_flag)) break;
        tc_fence_after();
        const uint32_t tsm = smem_u32(tmp_base + tb * Cfg::kTmpBytes);
        const uint32_t bsm = smem_u32(bst_base + st * Cfg::kBStageStride);
#pragma unroll
        for (int ks = 0; ks < RP / 16; ++ks) {
          const uint64_t adesc = smem_desc(tsm + ks * 256, 128, RP * 16, kSwizzleNone);
          const uint64_t bdesc = smem_desc(bsm + ks * 2048, Cfg::kBoxBytes, 1024, kSwizzle128);
          umma_f16(tmem_base + ab * kExpandNT, adesc, bdesc, idesc, ks != 0);
        }
        umma_commit(&bempty[st]);
        umma_commit(&afull[ab]);
        issued = true;
        ++bctr;
        ++unit_ctr;
      }
      if (issued) {
        umma_commit(drain);
        mbar_drain(drain, 0);
      }
    }
  } else if (warp == 2) {
    // ---------------- tmp gather: item rows -> K-major (no swizzle) tile
    uint32_t item_ctr = 0;
    int64_t prev = -1;
    while (units.next(tab, u)) {
      const int rank = tab.rk[u.slot];
      if (rank <= 0 || u.item_start == prev) continue;
      prev = u.item_start;
      const int tb = item_ctr & 1;
      if (!mbar_wait(&tempty[tb], ((item_ctr >> 1) & 1) ^ 1, abort_flag)) break;
      const int kr = min(rank, args.R);
      const uint32_t tbuf = smem_u32(tmp_base + tb * Cfg::kTmpBytes);
#pragma unroll
      for (int rr = 0; rr < kTileM / 32; ++rr) {
        const int r = lane + 32 * rr;
        if (r < u.cnt) {
          const uint8_t* src =
              args.tmp + (int64_t)__ldg(args.seg.token_index + u.item_start + r) * args.R * 2;
#pragma unroll
          for (int c = 0; c < RP / 8; ++c) {
            const int kleft = kr - c * 8;
            const uint32_t bytes = kleft >= 8 ? 16u : (kleft > 0 ? (uint32_t)kleft * 2u : 0u);
            const uint32_t dst = tbuf + (r >> 3) * (RP * 16) + c * 128 + (r & 7) * 16;
            cp_async_16(dst, bytes ? src + c * 16 : src, bytes);
          }
        }
      }
      cp_async_arrive_noinc(&tfull[tb]);
      ++item_ctr;
    }
    cp_async_wait_all();
  } else if (warp >= 4 && warp < 8) {
    // ---------------- TMEM readers: scaled, rounded delta rows -> smem
    const int q = warp & 3;       // TMEM lane quarter
    const int r = q * 32 + lane;  // token row of the item
    uint32_t unit_ctr = 0;
    while (units.next(tab, u)) {
      if (tab.rk[u.slot] <= 0) continue;
      const float scale = tab.sc[u.slot];
      const int ab = unit_ctr & 1;
      const uint32_t ph = (unit_ctr >> 1) & 1;
      if (!mbar_wait_warp(&afull[ab], ph, abort_flag)) break;
      if (!mbar_wait_warp(&dempty[ab], ph ^ 1, abort_flag)) break;
      tc_fence_after();
      const uint32_t drow = smem_u32(d_base + ab * Cfg::kDeltaBytes) + r * kDeltaRowBytes;
#pragma unroll
      for (int qc = 0; qc < kExpandNT / 32; ++qc) {
        uint32_t acc[2][16];
        const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + ab * kExpandNT + qc * 32;
        tmem_ld16(taddr, acc[0]);
        tmem_ld16(taddr + 16, acc[1]);
        tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t w[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int j = c * 8 + 2 * i;
            const float a0 = scale * __uint_as_float(acc[j >> 4][j & 15]);
            const float a1 = scale * __uint_as_float(acc[(j + 1) >> 4][(j + 1) & 15]);
            w[i] = (uint32_t)E::from_f(a0) | ((uint32_t)E::from_f(a1) << 16);
          }
          asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(drow + qc * 64 + c * 16),
                       "r"(w[0]), "r"(w[1]), "r"(w[2]), "r"(w[3])
                       : "memory");
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&aempty[ab]);
        mbar_arrive(&dfull[ab]);
      }
      ++unit_ctr;
    }
  } else if (warp >= 8) {
    // ---------------- y streams
    const int sw = warp - 8;  // 0..15
    const int hr = 2 * sw + (lane >> 4);
    const int c = lane & 15;
    ExpandUnits pre = units;  // prefetch cursor, one active unit ahead
    int64_t p_item = -1;
    int32_t p_tok[4] = {0, 0, 0, 0};
    // issues the loads of the next active unit of `pre` into `set`
    auto prefetch = [&](YSet& set) -> bool {
      ExpandUnit pu;
      bool found = false;
      while (pre.next(tab, pu)) {
        if (tab.rk[pu.slot] > 0) {
          found = true;
          break;
        }
      }
      if (!found) return false;
      // lanes c = 0 and c = 8 own the two 128-byte lines of a row segment
      auto prefetch_tile = [&](int tile) {
        const int col = tile * kExpandNT + c * 8;
        if ((c & 7) == 0 && col < args.N) {
#pragma unroll
          for (int j = 0; j < 4; ++j)
            if (32 * j + hr < pu.cnt) prefetch_l2(args.y + ((int64_t)p_tok[j] * args.N + col) * 2);
        }
      };
      if (pu.item_start != p_item) {
        p_item = pu.item_start;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int r = 32 * j + hr;
          p_tok[j] = r < pu.cnt ? __ldg(args.seg.token_index + pu.item_start + r) : 0;
        }
        for (int a = 1; a < kExpandPrefetch; ++a) prefetch_tile(pu.tile + a);
      }
      prefetch_tile(pu.tile + kExpandPrefetch);
      set.n0 = pu.tile * kExpandNT;
      const bool piece = c * 8 < args.N - set.n0;  // N % 8 == 0: pieces are all-or-nothing
      set.mask = 0;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int r = 32 * j + hr;
        set.tok[j] = p_tok[j];
        if (piece && r >= pu.t0 && r < pu.t1) {
          set.mask |= 1u << j;
          set.v[j] = *reinterpret_cast<const uint4*>(args.y + ((int64_t)p_tok[j] * args.N + set.n0 + c * 8) * 2);
        }
      }
      return true;
    };
    // adds the delta tile of unit `unit_ctr` to `set` and stores it
    auto apply = [&](YSet& set, uint32_t unit_ctr) -> bool {
      const int db = unit_ctr & 1;
      if (!mbar_wait_warp(&dfull[db], (unit_ctr >> 1) & 1, abort_flag)) return false;
      const uint32_t dtile = smem_u32(d_base + db * Cfg::kDeltaBytes);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (set.mask & (1u << j)) {
          const int r = 32 * j + hr;
          uint32_t d[4];
          asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                       : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
                       : "r"(dtile + r * kDeltaRowBytes + c * 16));
          uint32_t yv[4] = {set.v[j].x, set.v[j].y, set.v[j].z, set.v[j].w};
          uint32_t o[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float y0 = E::to_f((uint16_t)(yv[i] & 0xFFFFu)) + E::to_f((uint16_t)(d[i] & 0xFFFFu));
            const float y1 = E::to_f((uint16_t)(yv[i] >> 16)) + E::to_f((uint16_t)(d[i] >> 16));
            o[i] = (uint32_t)E::from_f(y0) | ((uint32_t)E::from_f(y1) << 16);
          }
          *reinterpret_cast<uint4*>(args.y + ((int64_t)set.tok[j] * args.N + set.n0 + c * 8) * 2) =
              make_uint4(o[0], o[1], o[2], o[3]);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&dempty[db]);
      return true;
    };
    YSet s0, s1;
    uint32_t unit_ctr = 0;
    bool have = prefetch(s0);
    while (have) {
      bool more = prefetch(s1);
      if (!apply(s0, unit_ctr++)) break;
      if (!more) break;
      have = prefetch(s0);
      if (!apply(s1, unit_ctr++)) break;
    }
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::kTmemCols);
  }
}

}  // namespace plora
