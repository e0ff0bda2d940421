// SGMV shrink and expand on the tensor cores with the token rows streamed
// straight into registers (mma.sync m16n8k16, bf16/fp16 in, fp32 accumulate).
//
// Both kernels are gathers over HBM with a tiny rank-R contraction: the shrink
// reads every active token's K-wide row of x once, the expand reads and
// rewrites its N-wide row of y once.  Their speed is set by how many bytes each
// SM keeps in flight and how few instructions and synchronisation points they
// spend per byte, so the token rows never pass through shared memory: each
// lane loads 16 bytes (8 consecutive columns of one token row) and those
// registers feed the mma directly; the expand writes its result back from
// registers too.  Only the slot's LoRA weights are staged in shared memory, in
// double-buffered 64 KB windows that TMA lands swizzled so that ldmatrix.trans
// reads them without bank conflicts.
//
// Work split: a CTA takes a contiguous share of the slot-ordered token list,
// cut into items of <= 128 tokens of one slot.  An item is 16-token tiles x
// K ranges (shrink) or N ranges (expand), one (tile, range) pair per warp.
// Window w + 2 of the CTA's window sequence is issued by the last warp to
// release window w.
//
// Reference semantics: src/polylora/sgmv.py:63-138 (_sgmv_lora_a_kernel) and
// sgmv.py:178-275 (_sgmv_lora_b_kernel).
#pragma once

#include "sgmv_common.cuh"

namespace plora {

constexpr int kMmaWarps = 16;                      // compute warps
constexpr int kMmaThreads = kMmaWarps * 32;
constexpr int kWinBoxRows = 256;                   // rows per weight TMA box (8 blocks of 32)

constexpr int kWinBufs = 2;           // LoRA weight windows in flight
constexpr int kWinBytes = 64 * 1024;  // one LoRA weight window

template <int RP>
struct ShrinkMmaCfg {
  static constexpr int kWinRows = kWinBytes / (RP * 2);  // K rows per window
  static constexpr int kBoxBytes = kWinBoxRows * RP * 2;
  // 32-column blocks per load batch (two batches alternate); larger batches
  // spill at the 128-register budget of 16 warps and measured slower
  static constexpr int kU = RP == 16 ? 4 : (RP == 32 ? 3 : 2);
  static constexpr int kPartBytes = kMmaWarps * 16 * RP * 4;    // one 16 x RP fp32 tile per warp
  static constexpr int kBarrierBytes = 64;
  // + slot table (3 * num_slots + 1 ints), sized at launch
  static constexpr int kSmemBytes = 1024 + kWinBufs * kWinBytes + kPartBytes + kBarrierBytes;
};

// 4x4 transpose of 32-bit words across the four lanes of a quad: lane t
// holds w[i] = M[t][i] on entry and M[i][t] on exit.
__device__ __forceinline__ void quad_transpose(uint32_t (&w)[4], int t) {
  const bool hi = t & 2;
  uint32_t s0 = hi ? w[0] : w[2], s1 = hi ? w[1] : w[3];
  uint32_t r0 = __shfl_xor_sync(0xffffffffu, s0, 2), r1 = __shfl_xor_sync(0xffffffffu, s1, 2);
  if (hi) {
    w[0] = r0;
    w[1] = r1;
  } else {
    w[2] = r0;
    w[3] = r1;
  }
  const bool odd = t & 1;
  s0 = odd ? w[0] : w[1];
  s1 = odd ? w[2] : w[3];
  r0 = __shfl_xor_sync(0xffffffffu, s0, 1);
  r1 = __shfl_xor_sync(0xffffffffu, s1, 1);
  if (odd) {
    w[0] = r0;
    w[2] = r1;
  } else {
    w[1] = r0;
    w[3] = r1;
  }
}

// 16-byte streaming load that does not allocate in L1 (rows are read once).
__device__ __forceinline__ uint4 ld_stream16(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

// Round-to-nearest add of two packed pairs of bf16 (BF16) or fp16 values.
template <bool BF16>
__device__ __forceinline__ uint32_t add2(uint32_t a, uint32_t b) {
  uint32_t r;
  if constexpr (BF16)
    asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  else
    asm("add.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

// Packs two floats (lo, hi) into a pair of bf16 (BF16) or fp16, round to nearest.
template <bool BF16>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  uint32_t r;
  if constexpr (BF16)
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  else
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

// Four 8x8 matrices of 16-bit pairs from mma fragment layout to shared memory
// (lane l gives the address of row l & 7 of matrix l >> 3).
__device__ __forceinline__ void stsm_x4(uint32_t addr, const uint32_t (&r)[4]) {
  asm volatile("stmatrix.sync.aligned.m8n8.x4.shared.b16 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(r[0]),
               "r"(r[1]), "r"(r[2]), "r"(r[3])
               : "memory");
}

__device__ __forceinline__ void lds_v4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr)
               : "memory");
}

// d += a (16x16, row) * b (16x8, col); fp32 accumulate.
template <bool BF16>
__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                          uint32_t b1) {
  if constexpr (BF16) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
        "{%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
        "{%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
}

// Shared-memory byte offset of 16-byte chunk j of row position k of a weight
// window written by TMA with the swizzle that matches its row width (32/64/128
// B for RP = 16/32/64): the chunk index is XORed with address bits 7 and up.
// Within a 32-row block, position 8 cc + 2 m + e holds weight row 8 m + 2 cc + e.
template <int RP>
__device__ __forceinline__ uint32_t win_offset(int k, int j) {
  constexpr int kRowBytes = RP * 2;
  const uint32_t off = (uint32_t)k * kRowBytes;
  return off + 16u * ((uint32_t)j ^ ((off >> 7) & (RP / 8 - 1)));
}

// Issues one LoRA-A window: nb 32-row blocks from block blk0 of the 5-D view,
// 8-block boxes then single blocks (one thread; out of line: the shrink has
// one release site per unrolled block).
__device__ __noinline__ void issue_lora_a_window(const CUtensorMap* map8, const CUtensorMap* map1,
                                                 uint64_t* bar, uint32_t dst, int nb, int blk0,
                                                 int block_bytes) {
  mbar_arrive_expect_tx(bar, nb * block_bytes);
  int q = 0;
  for (; q + 8 <= nb; q += 8) tma_load_5d_outer(dst + q * block_bytes, map8, bar, blk0 + q);
  for (; q < nb; ++q) tma_load_5d_outer(dst + q * block_bytes, map1, bar, blk0 + q);
}

// Sequence of the weight windows of the CTA's work (slot, window), in
// the order every warp consumes them.
template <class WorkIt>
struct WinCursor {
  WorkIt it;
  int slot, w, w_hi;
  bool valid;
  __device__ void init(const SlotTab& tab, const WorkIt& src) {
    it = src;
    w_hi = -1;
    w = 0;
    valid = true;
    advance(tab);
  }
  // out-of-line copy for kernels whose many release sites would otherwise each
  // carry one (measured faster in the shrink, slower in the expand)
  __device__ __noinline__ void advance_outlined(const SlotTab& tab) { advance(tab); }
  __device__ __forceinline__ void advance(const SlotTab& tab) {
    if (++w <= w_hi) return;
    Work nx;
    if (it.next(tab, nx)) {
      slot = nx.slot;
      w = nx.w_lo;
      w_hi = nx.w_hi;
      return;
    }
    valid = false;
  }
};

// Bytes of the staged slot table (3 * ns + 1 ints, 16-byte aligned).
__host__ __device__ constexpr int64_t slot_tab_bytes(int64_t ns) { return ((3 * ns + 1) * 4 + 15) & ~15ll; }

// tmp[t, :] = x[t, :] @ A[slot(t)] for the active tokens of the table.
// 16 warps; an item is 16-token tiles x K ranges, one pair per warp.  The
// slot's LoRA-A rows stream through two 64 KB windows: windows 0 and 1 are
// issued at start, and the last warp to release window c issues c + 2.
template <int RP, bool BF16>
__global__ void __launch_bounds__(kMmaThreads, 1)
    sgmv_shrink_mma_kernel(const __grid_constant__ CUtensorMap tmap_a8,
                           const __grid_constant__ CUtensorMap tmap_a1, const ShrinkArgs args) {
  using WorkIt = TokenWork;
  using Cfg = ShrinkMmaCfg<RP>;
  using E = Elem<BF16>;
  constexpr int W = Cfg::kWinRows;
  constexpr int NB = kWinBufs;
  constexpr int U = Cfg::kU;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  float* part = reinterpret_cast<float*>(smem + NB * kWinBytes);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + NB * kWinBytes + Cfg::kPartBytes);
  uint32_t* released = reinterpret_cast<uint32_t*>(full + NB);  // per buffer, monotonic
  volatile int* abort_flag = reinterpret_cast<volatile int*>(released + NB);
  uint32_t* issued = reinterpret_cast<uint32_t*>(released + NB) + 1;  // per buffer: windows issued into it
  int32_t* tab_mem =
      reinterpret_cast<int32_t*>(smem + NB * kWinBytes + Cfg::kPartBytes + Cfg::kBarrierBytes);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  griddep_wait();    // inputs (segment table, x) come from earlier kernels
  griddep_launch();  // the expand may start on SMs this grid releases
  const int64_t total = ld_cg_i32(args.seg.slot_start + args.seg.num_slots);
  const int64_t begin = total * blockIdx.x / gridDim.x;
  const int64_t end = total * (blockIdx.x + 1) / gridDim.x;
  if (begin >= end) return;  // uniform across the CTA

  const SlotTab tab = stage_slot_tab(args.seg, args.ranks, nullptr, tab_mem);
  const int K = args.K;
  const int nwin = (K + W - 1) / W;
  const int kblocks = K >> 5;  // 32-row blocks per slot
  auto issue = [&](const WinCursor<WorkIt>& wc, int b) {  // one thread
    atomicAdd(&issued[b], 1u);
    issue_lora_a_window(&tmap_a8, &tmap_a1, &full[b], smem_u32(smem + b * kWinBytes),
                        min(W, K - wc.w * W) >> 5, wc.slot * kblocks + wc.w * (W >> 5), 32 * RP * 2);
  };
  __syncthreads();  // slot table staged
  WorkIt work;
  work.init(tab, begin, end, nwin);
  WinCursor<WorkIt> ic;  // the window this warp would issue after its next release
  ic.init(tab, work);
  if (threadIdx.x == 0) {
    for (int i = 0; i < NB; ++i) {
      mbar_init(&full[i], 1);
      released[i] = 0;
      issued[i] = 0;
    }
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tmap(&tmap_a8);
    prefetch_tmap(&tmap_a1);
    for (int b = 0; b < NB && ic.valid; ++b) {
      issue(ic, b);
      ic.advance_outlined(tab);
    }
  } else {
    for (int b = 0; b < NB; ++b) ic.advance(tab);
  }
  __syncthreads();

  const int g = lane >> 2;  // fragment row group
  const int t = lane & 3;   // lane within the quad
  const uint32_t win_base = smem_u32(smem);
  uint32_t c_base = 0;  // window counter at the start of the item
  bool ok = true;
  Work wk;
  while (work.next(tab, wk)) {
    const int s = wk.slot;
    const int64_t start = wk.start;
    const int cnt = wk.cnt;
    const int rank = tab.rk[s];
    const int tiles = (cnt + 15) >> 4;
    const int KS = max(1, kMmaWarps / tiles);
    const bool active = warp < tiles * KS;
    const int tile = active ? warp / KS : 0;
    const int ks = active ? warp - tile * KS : 0;
    const int r0 = tile * 16 + g;
    const bool v0 = active && r0 < cnt, v1 = active && r0 + 8 < cnt;
    const uint8_t* x0 = args.x + (v0 ? (int64_t)ld_cg_i32(args.seg.token_index + start + r0) : 0) * K * 2;
    const uint8_t* x1 = args.x + (v1 ? (int64_t)ld_cg_i32(args.seg.token_index + start + r0 + 8) : 0) * K * 2;

    // this warp's 32-column blocks of window w: [b0, b1); cursors over
    // (window, block) skip windows without blocks
    struct Cur {
      int w, blk, end;
    };
    auto range = [&](Cur& c) {
      const int nb = (min(W, K - c.w * W) + 31) >> 5;
      c.blk = active ? ks * nb / KS : 0;
      c.end = active ? (ks + 1) * nb / KS : 0;
    };
    auto first = [&](Cur& c) {
      c.w = 0;
      range(c);
      while (c.blk >= c.end && ++c.w < nwin) range(c);
    };
    auto step = [&](Cur& c) {
      if (++c.blk >= c.end)
        while (++c.w < nwin) {
          range(c);
          if (c.blk < c.end) break;
        }
    };
    Cur lc, mc;  // load cursor, compute cursor (same sequence)
    first(lc);
    first(mc);

    struct Batch {
      uint4 x0[U], x1[U];
    };
    auto load_batch = [&](Batch& B) {
#pragma unroll
      for (int u = 0; u < U; ++u) {
        if (lc.w < nwin) {
          const int col = lc.w * W + lc.blk * 32 + 8 * t;
          const bool in = col < K;
          B.x0[u] = (v0 && in) ? ld_stream16(x0 + col * 2) : make_uint4(0u, 0u, 0u, 0u);
          B.x1[u] = (v1 && in) ? ld_stream16(x1 + col * 2) : make_uint4(0u, 0u, 0u, 0u);
          step(lc);
        }
      }
    };

    float acc[RP / 16][2][4];  // D^T tiles: rank rows 16 rt .., tokens 8 nt ..
#pragma unroll
    for (int rt = 0; rt < RP / 16; ++rt)
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) acc[rt][nt][0] = acc[rt][nt][1] = acc[rt][nt][2] = acc[rt][nt][3] = 0.f;
    int cw = -1;  // window of this item the warp currently holds
    // releases the held window; the last of the 16 releasers refills its buffer
    auto release = [&]() {
      const uint32_t b = (c_base + cw) % NB;
      __syncwarp();
      if (lane == 0) {
        __threadfence_block();
        if (atomicAdd(&released[b], 1u) % kMmaWarps == kMmaWarps - 1 && ic.valid && !*abort_flag) {
          fence_proxy_async_smem();
          issue(ic, b);
        }
      }
      ic.advance(tab);
    };
    // moves the hold forward to window `to` of the item
    auto hold = [&](int to) {
      while (cw < to) {
        if (cw >= 0) release();
        ++cw;
        const uint32_t c = c_base + cw;
        if (ok) ok = mbar_wait_warp(&full[c % NB], (c / NB) & 1, abort_flag);
      }
    };
    auto compute_batch = [&](Batch& B) {
#pragma unroll
      for (int u = 0; u < U; ++u) {
        if (mc.w >= nwin) break;
        hold(mc.w);
        // B fragments of k16 step s: tokens g (x0) and 8 + g (x1), k = 8t + 4s + {0,1} / {2,3}
        const uint32_t fb0[2][2] = {{B.x0[u].x, B.x0[u].y}, {B.x0[u].z, B.x0[u].w}};
        const uint32_t fb1[2][2] = {{B.x1[u].x, B.x1[u].y}, {B.x1[u].z, B.x1[u].w}};
        const uint32_t wb = win_base + ((c_base + mc.w) % NB) * kWinBytes;
        const int mi = lane >> 3;
#pragma unroll
        for (int st = 0; st < 2; ++st) {
          const int pos = mc.blk * 32 + (2 * st + (mi >> 1)) * 8 + (lane & 7);
#pragma unroll
          for (int rt = 0; rt < RP / 16; ++rt) {
            uint32_t fa[4];
            ldsm_x4_trans(wb + win_offset<RP>(pos, 2 * rt + (mi & 1)), fa);
            if (ok) {
              mma_16816<BF16>(acc[rt][0], fa, fb0[st][0], fb0[st][1]);
              mma_16816<BF16>(acc[rt][1], fa, fb1[st][0], fb1[st][1]);
            }
          }
        }
        step(mc);
      }
    };

    Batch A, B;
    load_batch(A);
    for (;;) {
      const bool more_b = lc.w < nwin;
      if (more_b) load_batch(B);
      compute_batch(A);
      if (!more_b) break;
      const bool more_a = lc.w < nwin;
      if (more_a) load_batch(A);
      compute_batch(B);
      if (!more_a) break;
    }
    hold(nwin - 1);  // windows without blocks of this warp are passed through
    release();
    c_base += nwin;

    // partial sums -> shared memory -> reduced, rounded rows of tmp
    if (active) {  // part[warp][token 0..15][rank]
      float* p = part + (size_t)warp * 16 * RP;
#pragma unroll
      for (int rt = 0; rt < RP / 16; ++rt)
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
          const int tk = 8 * nt + 2 * t, r = 16 * rt + g;
          p[tk * RP + r] = acc[rt][nt][0];
          p[(tk + 1) * RP + r] = acc[rt][nt][1];
          p[tk * RP + r + 8] = acc[rt][nt][2];
          p[(tk + 1) * RP + r + 8] = acc[rt][nt][3];
        }
    }
    named_barrier(1, kMmaWarps * 32);
    const int n_eff = min(rank * args.stack_num, args.R);
    for (int u = threadIdx.x; u < tiles * 16 * (RP / 8); u += kMmaWarps * 32) {
      const int row = u / (RP / 8), cg = u - row * (RP / 8);
      if (row >= cnt) continue;
      const int tl = row >> 4, rr = row & 15;
      float v[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = 0.f;
      for (int q = 0; q < KS; ++q) {
        const float* p = part + ((size_t)(tl * KS + q) * 16 + rr) * RP + cg * 8;
        const float4 lo = *reinterpret_cast<const float4*>(p);
        const float4 hi = *reinterpret_cast<const float4*>(p + 4);
        v[0] += lo.x; v[1] += lo.y; v[2] += lo.z; v[3] += lo.w;
        v[4] += hi.x; v[5] += hi.y; v[6] += hi.z; v[7] += hi.w;
      }
      uint32_t o[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int c0 = cg * 8 + 2 * i;
        o[i] = (uint32_t)E::from_f(c0 < n_eff ? v[2 * i] : 0.f) |
               ((uint32_t)E::from_f(c0 + 1 < n_eff ? v[2 * i + 1] : 0.f) << 16);
      }
      const int64_t tok = ld_cg_i32(args.seg.token_index + start + row);
      *reinterpret_cast<uint4*>(args.tmp + (tok * args.R + cg * 8) * 2) = make_uint4(o[0], o[1], o[2], o[3]);
    }
    named_barrier(1, kMmaWarps * 32);
  }
  // the last window issued into each buffer has landed (unless a wait gave up
  // early; no window is issued after that), so no copy writes this CTA's
  // shared memory after it exits
  __syncthreads();
  if (threadIdx.x == 0)
    for (int b = 0; b < NB; ++b)
      if (issued[b]) mbar_drain(&full[b], (issued[b] - 1u) & 1u);
}

// ============================================================== expand
// y[t, :] += round(scale * tmp[t, :] @ B[slot(t)]) in place, with the
// reference's rounding order (the fp32 product is scaled and rounded to the
// activation type, then added to the base output and rounded again).
//
// The y rows are the only large stream (read and written once), so they stay
// in registers: a lane loads 16 bytes (8 consecutive columns) of a token row,
// the mma.sync D fragments of the matching 32-column block are rounded, packed
// and regrouped across the lane quad so that each lane holds the delta of its
// own 8 columns, added, and stored back.  tmp rows (R values per token) are
// loaded once per tile as A fragments; the slot's LoRA-B rows stream through
// 64 KB windows (a 4-D TMA view lands 64-column chunks of all R rows, 128-byte
// swizzled, so ldmatrix.trans reads them without bank conflicts).
//
// Work split: as the shrink, items of <= 128 tokens of one slot inside the
// CTA's token share; an item is 16-token tiles x column ranges of each window.
//
// Reference semantics: src/polylora/sgmv.py:178-275 (_sgmv_lora_b_kernel).
template <int RP>
struct ExpandMmaCfg {
  static constexpr int kWinCols = kWinBytes / (RP * 2);  // N columns per window
  static constexpr int kChunkBytes = RP * 128;           // 64 columns x RP rows
  static constexpr int kBoxChunks = kWinCols / 64 < 16 ? kWinCols / 64 : 16;
  static constexpr int kU = RP == 64 ? 2 : 3;            // 32-column blocks per load batch
  static constexpr int kBarrierBytes = 64;
  // 64-byte delta rows; 16-byte chunk j of row r sits at chunk j ^ ((r >> 1) & 3), so
  // both the stmatrix rows and the lanes' 16-byte reads hit 8 distinct bank groups
  static constexpr int kRegroupPitch = 64;
  static constexpr int kRegroupBytes = kMmaWarps * 16 * kRegroupPitch;
  // + slot table (3 * num_slots + 1 ints), sized at launch
  static constexpr int kSmemBytes = 1024 + kWinBufs * kWinBytes + kBarrierBytes + kRegroupBytes;
};

template <int RP, bool BF16>
__global__ void __launch_bounds__(kMmaThreads, 1)
    sgmv_expand_mma_kernel(const __grid_constant__ CUtensorMap tmap_bn,
                           const __grid_constant__ CUtensorMap tmap_b1, const ExpandArgs args) {
  using WorkIt = TokenWork;
  using Cfg = ExpandMmaCfg<RP>;
  constexpr int NB = kWinBufs;
  using E = Elem<BF16>;
  constexpr int W = Cfg::kWinCols;
  constexpr int U = Cfg::kU;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + NB * kWinBytes);
  uint32_t* released = reinterpret_cast<uint32_t*>(full + NB);  // per buffer, monotonic
  volatile int* abort_flag = reinterpret_cast<volatile int*>(released + NB);
  uint32_t* issued = reinterpret_cast<uint32_t*>(released + NB) + 1;  // per buffer: windows issued into it
  uint8_t* regroup = smem + NB * kWinBytes + Cfg::kBarrierBytes;  // per-warp 16 x 64 B delta tile
  int32_t* tab_mem = reinterpret_cast<int32_t*>(regroup + Cfg::kRegroupBytes);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t total = ld_cg_i32(args.seg.slot_start + args.seg.num_slots);
  const int64_t begin = total * blockIdx.x / gridDim.x;
  const int64_t end = total * (blockIdx.x + 1) / gridDim.x;
  if (begin >= end) return;  // uniform across the CTA

  const SlotTab tab = stage_slot_tab(args.seg, args.ranks, args.scales, tab_mem);
  const int N = args.N;
  const int nwin = (N + W - 1) / W;
  auto issue = [&](const WinCursor<WorkIt>& wc, int b) {  // one thread
    atomicAdd(&issued[b], 1u);
    const int nc = min(W, N - wc.w * W) >> 6;
    mbar_arrive_expect_tx(&full[b], nc * Cfg::kChunkBytes);
    const int ch0 = wc.w * (W >> 6);
    const uint32_t dst = smem_u32(smem + b * kWinBytes);
    int q = 0;
    for (; q + Cfg::kBoxChunks <= nc; q += Cfg::kBoxChunks)
      tma_load_4d_outer(dst + q * Cfg::kChunkBytes, &tmap_bn, &full[b], ch0 + q, wc.slot);
    for (; q < nc; ++q)
      tma_load_4d_outer(dst + q * Cfg::kChunkBytes, &tmap_b1, &full[b], ch0 + q, wc.slot);
  };
  __syncthreads();  // slot table staged
  WorkIt work;
  work.init(tab, begin, end, nwin);
  WinCursor<WorkIt> ic;  // the window this warp would issue after its next release
  ic.init(tab, work);
  if (threadIdx.x == 0) {
    for (int i = 0; i < NB; ++i) {
      mbar_init(&full[i], 1);
      released[i] = 0;
      issued[i] = 0;
    }
    *abort_flag = 0;
    fence_barrier_init();
    prefetch_tmap(&tmap_bn);
    prefetch_tmap(&tmap_b1);
    for (int b = 0; b < NB && ic.valid; ++b) {
      issue(ic, b);
      ic.advance(tab);
    }
  } else {
    for (int b = 0; b < NB; ++b) ic.advance(tab);
  }
  __syncthreads();

  const int g = lane >> 2;  // fragment row group
  const int t = lane & 3;   // lane within the quad
  const uint32_t win_base = smem_u32(smem);
  uint32_t c_base = 0;  // window counter at the start of the work
  bool ok = true;
  Work wk;
  while (work.next(tab, wk)) {
    const int s = wk.slot;
    const int64_t start = wk.start;
    const int cnt = wk.cnt;
    const int wlo = wk.w_lo, whi = wk.w_hi;  // this work's windows
    const int rank = tab.rk[s];
    const float scale = tab.sc[s];
    const int tiles = (cnt + 15) >> 4;
    const int CS = max(1, kMmaWarps / tiles);
    const bool active = warp < tiles * CS;
    const int tile = active ? warp / CS : 0;
    const int cs = active ? warp - tile * CS : 0;
    const int r0 = tile * 16 + g;
    const bool v0 = active && r0 < cnt, v1 = active && r0 + 8 < cnt;
    const int64_t tok0 = v0 ? (int64_t)ld_cg_i32(args.seg.token_index + start + r0) : 0;
    const int64_t tok1 = v1 ? (int64_t)ld_cg_i32(args.seg.token_index + start + r0 + 8) : 0;
    uint8_t* y0 = args.y + tok0 * N * 2;
    uint8_t* y1 = args.y + tok1 * N * 2;

    uint32_t fa[RP / 16][4];  // A fragments (tmp rows), filled once the first y batch is in flight

    struct Cur {
      int w, blk, end;
    };
    auto range = [&](Cur& c) {
      const int nb = min(W, N - c.w * W) >> 5;
      c.blk = active ? cs * nb / CS : 0;
      c.end = active ? (cs + 1) * nb / CS : 0;
    };
    auto first = [&](Cur& c) {
      c.w = wlo;
      range(c);
      while (c.blk >= c.end && ++c.w <= whi) range(c);
    };
    auto step = [&](Cur& c) {
      if (++c.blk >= c.end)
        while (++c.w <= whi) {
          range(c);
          if (c.blk < c.end) break;
        }
    };
    Cur lc, mc;  // load cursor, compute cursor (same sequence)
    first(lc);
    first(mc);

    struct Batch {
      uint4 y0[U], y1[U];
    };
    auto load_batch = [&](Batch& B) {
#pragma unroll
      for (int u = 0; u < U; ++u) {
        if (lc.w <= whi) {
          const int col = lc.w * W + lc.blk * 32 + 8 * t;
          B.y0[u] = v0 ? ld_stream16(y0 + col * 2) : make_uint4(0u, 0u, 0u, 0u);
          B.y1[u] = v1 ? ld_stream16(y1 + col * 2) : make_uint4(0u, 0u, 0u, 0u);
          step(lc);
        }
      }
    };

    int cw = wlo - 1;  // window of this work the warp currently holds
    auto release = [&]() {
      const uint32_t b = (c_base + cw - wlo) % NB;
      __syncwarp();
      if (lane == 0) {
        __threadfence_block();
        if (atomicAdd(&released[b], 1u) % kMmaWarps == kMmaWarps - 1 && ic.valid && !*abort_flag) {
          fence_proxy_async_smem();
          issue(ic, b);
        }
      }
      ic.advance(tab);
    };
    auto hold = [&](int to) {
      while (cw < to) {
        if (cw >= wlo) release();
        ++cw;
        const uint32_t c = c_base + cw - wlo;
        if (ok) ok = mbar_wait_warp(&full[c % NB], (c / NB) & 1, abort_flag);
      }
    };
    // y + delta for the 8 columns of a lane: words hold bf16/fp16 pairs
    // (a correctly rounded pair add equals the fp32 add rounded once: the fp32
    // sum of two 16-bit floats is exact unless one addend is below half an ulp)
    auto add_store = [&](uint8_t* row, bool v, int col, const uint4& yv, const uint32_t (&d)[4]) {
      const uint4 o = make_uint4(add2<BF16>(yv.x, d[0]), add2<BF16>(yv.y, d[1]), add2<BF16>(yv.z, d[2]),
                                 add2<BF16>(yv.w, d[3]));
      if (v) *reinterpret_cast<uint4*>(row + col * 2) = o;
    };
    // stmatrix: lane l writes row l & 7 of matrix (tile) l >> 3; ld: row g, columns 8t ..
    const uint32_t rg_base = smem_u32(regroup + warp * 16 * Cfg::kRegroupPitch);
    const uint32_t rg_st =
        rg_base + (lane & 7) * Cfg::kRegroupPitch + 16 * ((lane >> 3) ^ (((lane & 7) >> 1) & 3));
    const uint32_t rg_ld = rg_base + g * Cfg::kRegroupPitch + 16 * (t ^ ((g >> 1) & 3));
    auto compute_batch = [&](Batch& B) {
#pragma unroll
      for (int u = 0; u < U; ++u) {
        if (mc.w > whi) break;
        hold(mc.w);
        const uint32_t wb = win_base + ((c_base + mc.w - wlo) % NB) * kWinBytes;
        const int cwin = mc.blk * 32;  // block column inside the window
        float acc[4][4];
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
        const int m = lane >> 3;  // ldmatrix matrix of this lane: tile jb + (m >> 1), k half m & 1
#pragma unroll
        for (int st = 0; st < RP / 16; ++st) {
#pragma unroll
          for (int jb = 0; jb < 4; jb += 2) {
            const int c0 = cwin + 8 * (jb + (m >> 1));
            const int k = 16 * st + 8 * (m & 1) + (lane & 7);
            const uint32_t addr = wb + (c0 >> 6) * Cfg::kChunkBytes + k * 128 +
                                  16 * (((c0 >> 3) & 7) ^ (k & 7));
            uint32_t bf[4];
            ldsm_x4_trans(addr, bf);
            if (ok) {
              mma_16816<BF16>(acc[jb], fa[st], bf[0], bf[1]);
              mma_16816<BF16>(acc[jb + 1], fa[st], bf[2], bf[3]);
            }
          }
        }
        // delta words (tile j, row g / g + 8), regrouped to the lane's 8 columns
        uint32_t d0[4], d1[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          d0[j] = pack2<BF16>(scale * acc[j][0], scale * acc[j][1]);
          d1[j] = pack2<BF16>(scale * acc[j][2], scale * acc[j][3]);
        }
        // the D fragments are 8x8 tiles (rows g / g + 8, columns 8 j ..): stored
        // as matrices and read back as the lane's 16-byte row piece
        stsm_x4(rg_st, d0);
        stsm_x4(rg_st + 8 * Cfg::kRegroupPitch, d1);
        __syncwarp();
        lds_v4(rg_ld, d0);
        lds_v4(rg_ld + 8 * Cfg::kRegroupPitch, d1);
        __syncwarp();
        const int col = mc.w * W + cwin + 8 * t;
        add_store(y0, v0 && ok, col, B.y0[u], d0);
        add_store(y1, v1 && ok, col, B.y1[u], d1);
        step(mc);
      }
    };

    Batch A, B;
    load_batch(A);
    // tmp is the previous kernel's output: everything above (slot table, LoRA-B
    // windows, the first y batch) may overlap its tail under programmatic launch
    griddep_wait();
    // A fragments: tmp rows of this tile, columns >= min(rank, R) read as zero
    {
      const int kr = min(rank, args.R);
      const uint8_t* t0 = args.tmp + tok0 * args.R * 2;
      const uint8_t* t1 = args.tmp + tok1 * args.R * 2;
      auto ld2 = [&](const uint8_t* row, bool v, int k) -> uint32_t {
        if (!v || k >= kr) return 0u;
        const uint32_t w = ld_ca_u32(row + k * 2);
        return k + 1 < kr ? w : (w & 0xFFFFu);
      };
#pragma unroll
      for (int st = 0; st < RP / 16; ++st) {
        fa[st][0] = ld2(t0, v0, 16 * st + 2 * t);
        fa[st][1] = ld2(t1, v1, 16 * st + 2 * t);
        fa[st][2] = ld2(t0, v0, 16 * st + 8 + 2 * t);
        fa[st][3] = ld2(t1, v1, 16 * st + 8 + 2 * t);
      }
    }
    for (;;) {
      const bool more_b = lc.w <= whi;
      if (more_b) load_batch(B);
      compute_batch(A);
      if (!more_b) break;
      const bool more_a = lc.w <= whi;
      if (more_a) load_batch(A);
      compute_batch(B);
      if (!more_a) break;
    }
    hold(whi);  // windows without blocks of this warp are passed through
    release();
    c_base += whi - wlo + 1;
  }
  // the last window issued into each buffer has landed (unless a wait gave up
  // early; no window is issued after that), so no copy writes this CTA's
  // shared memory after it exits
  __syncthreads();
  if (threadIdx.x == 0)
    for (int b = 0; b < NB; ++b)
      if (issued[b]) mbar_drain(&full[b], (issued[b] - 1u) & 1u);
}

}  // namespace plora
