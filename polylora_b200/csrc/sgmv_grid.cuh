// SGMV shrink and expand for batches of few tokens per slot (decode): the
// slot grid.
//
// With a handful of tokens per LoRA slot the work is streaming each used
// slot's LoRA weights once.  The token-split kernels (one CTA per share of the
// token list, walking all of a slot's weight windows) are bound by that serial
// walk there; these kernels give every (slot, weight part) its own CTA, so the
// weights of all slots stream in parallel over the whole GPU:
//  * expand: grid (N / 512 column chunks, slots).  CTA (c, s) computes
//    y += round(scale tmp B[s]) for columns [512 c, 512 c + 512) of slot s's
//    tokens.  Each warp owns 64 columns: it copies those columns of the slot's
//    LoRA-B rows (only the first ceil(rank / 16) * 16) into its own shared
//    tile with cp.async once, then runs the mma for each 16-token tile of the
//    slot.  No barrier between warps.
//  * shrink: grid (KP K parts, slots), clusters of the KP parts of a slot.
//    CTA (q, s) accumulates x A[s] over the K rows of part q for each 16-token
//    tile of the slot; CTA 0 of the cluster adds the parts' fp32 partials in
//    part order through distributed shared memory, rounds and writes tmp.
// Grid rows are slots, plus rows for the later 16-token tiles of slots with
// more than 16 tokens (grid_row), while the rows fit a grid dimension.  Results are
// deterministic (fixed summation order).  The mma operands and shared-memory
// layouts are those of the token-split kernels (sgmv_mma.cuh).
//
// Reference semantics: src/polylora/sgmv.py:63-138 (_sgmv_lora_a_kernel) and
// sgmv.py:178-275 (_sgmv_lora_b_kernel).
#pragma once

#include "sgmv_mma.cuh"

namespace plora {

constexpr int kGridWarps = 8;
constexpr int kGridThreads = kGridWarps * 32;
constexpr int kGridTile = 16;               // tokens per mma tile
constexpr int kGridCols = 64 * kGridWarps;  // expand: columns per CTA, 64 per warp
constexpr int kGridRows = 64;               // shrink: K rows a warp stages at once (2 blocks)

template <int RP>
struct ExpandGridCfg {
  static constexpr int kStageBytes = RP * 128;  // 64 columns x RP rows of B
  static constexpr int kRegroupBytes = 16 * 64;
  static constexpr int kSmemBytes = 1024 + kGridWarps * (kStageBytes + kRegroupBytes);
};

template <int RP>
struct ShrinkGridCfg {
  static constexpr int kStageBytes = kGridRows * RP * 2;  // also holds the warp's 16 x RP fp32 partial
  static constexpr int kPartBytes = kGridTile * RP * 4;   // the CTA's partial tmp rows
  static constexpr int kSmemBytes = 1024 + kGridWarps * kStageBytes + kPartBytes;
};

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Barrier over the CTAs of the cluster.  Every CTA of a cluster reaches it:
// the shrink exits early only per slot, which a cluster shares.
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t cluster_map(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
__device__ __forceinline__ float4 ld_cluster_f4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

// Grid rows by 16-token tile (by_tile): the first num_tokens / 16 rows take the
// later tiles (tile >= 1) of slots of rank > 0, the e-th in slot order for row
// e, found by a warp scan of the slots' later-tile counts; row E + s (E =
// num_tokens / 16) takes the first tile of slot s, as one load round trip
// shows (slot_start, rank).  So a popular slot's tiles run in parallel in CTAs
// of their own, launched first, while a row of an empty slot still costs one
// round trip; only the few later-tile rows scan, and those past the last
// later tile leave after one warp reduction.  Warp-collective; false when the
// row has no tile.
struct GridTile {
  int slot, rank;
  int64_t begin, end;  // this row's tokens in the segment table
};

__device__ __forceinline__ bool grid_later_tile(const SegTable& seg, const int32_t* ranks, int e, int lane,
                                                GridTile& out) {
  int carry = 0;        // later tiles of the slots before this round
  bool found = false;   // warp-uniform
  for (int c0 = 0; c0 < seg.num_slots; c0 += 256) {
    int st[8], cnt[8], rk[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int sl = c0 + 32 * k + lane;
      st[k] = cnt[k] = rk[k] = 0;
      if (sl < seg.num_slots) {
        st[k] = ld_cg_i32(seg.slot_start + sl);
        cnt[k] = ld_cg_i32(seg.slot_start + sl + 1) - st[k];
        rk[k] = __ldg(ranks + sl);
      }
    }
    {  // rows past the last later tile (most of them) leave after one reduction
      int sum = 0;
#pragma unroll
      for (int k = 0; k < 8; ++k) sum += (rk[k] > 0 && cnt[k] > kGridTile) ? (cnt[k] - 1) / kGridTile : 0;
      const int total = __reduce_add_sync(0xffffffffu, sum);
      if (e >= carry + total) {
        carry += total;
        continue;
      }
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int nt = (rk[k] > 0 && cnt[k] > kGridTile) ? (cnt[k] - 1) / kGridTile : 0;
      int incl = nt;
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        const int u = __shfl_up_sync(0xffffffffu, incl, d);
        if (lane >= d) incl += u;
      }
      const int lo = carry + incl - nt;  // this lane's slot's first later tile
      // no exit inside the unrolled loop: st/cnt/rk stay in registers
      const uint32_t hit = __ballot_sync(0xffffffffu, !found && lo <= e && e < lo + nt);
      if (hit != 0u) {
        const int l = __ffs(hit) - 1;
        const int tile = 1 + e - __shfl_sync(0xffffffffu, lo, l);
        const int64_t b = __shfl_sync(0xffffffffu, st[k], l);
        const int64_t n = __shfl_sync(0xffffffffu, cnt[k], l);
        out.slot = c0 + 32 * k + l;
        out.rank = __shfl_sync(0xffffffffu, rk[k], l);
        out.begin = b + (int64_t)kGridTile * tile;
        out.end = min(b + n, out.begin + kGridTile);
        found = true;
      }
      carry += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (found) return true;
  }
  return false;
}

// This CTA's row of the grid: a whole slot (!by_tile) or one tile of one.
__device__ __forceinline__ bool grid_row(const SegTable& seg, const int32_t* ranks, bool by_tile,
                                         int later_rows, int lane, GridTile& out) {
  const int j = (int)blockIdx.y - (by_tile ? later_rows : 0);
  if (j >= 0) {
    out.slot = j;
    out.begin = ld_cg_i32(seg.slot_start + j);
    out.end = ld_cg_i32(seg.slot_start + j + 1);
    out.rank = __ldg(ranks + j);
    if (by_tile) out.end = min(out.end, out.begin + kGridTile);
    return true;
  }
  return grid_later_tile(seg, ranks, (int)blockIdx.y, lane, out);
}

// Grid rows of the by-tile mapping for num_tokens tokens over num_slots slots:
// at most num_tokens / 16 later tiles, then one row per slot.  Which kernels
// take it (config-4 decode, 256 tokens over 128 slots, on B200): the shrink
// while its clusters have at most 8 K parts (q_proj 34.7 -> 26.8 us; with 16
// parts the extra 16-CTA cluster rows cost more than the split saved, 65.6 ->
// 68.8 us at K = 14336), the expand while it has at most 16 column chunks
// (q_proj 24.7 -> 18.3 us; at N = 14336 the grid is many waves deep and
// splitting cost 37.0 -> 42.9 us).
constexpr int kTileMaxKParts = 8;
constexpr int kTileMaxColChunks = 16;
__host__ __device__ inline int64_t grid_later_rows(int64_t num_tokens) { return num_tokens / kGridTile; }
__host__ __device__ inline int64_t grid_tile_rows(int64_t num_tokens, int64_t num_slots) {
  return grid_later_rows(num_tokens) + num_slots;
}

// ------------------------------------------------------------------- expand
template <int RP, bool BF16>
// 3 CTAs per SM (<= 85 registers, 75 KB of shared memory each at rank 64): at
// config-4 decode the gate_proj expand took 30.0 us against 36.9 with 2.
__global__ void __launch_bounds__(kGridThreads, 3)
    sgmv_expand_grid_kernel(const ExpandArgs args, bool by_tile, int later_rows) {
  using Cfg = ExpandGridCfg<RP>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // this CTA's tokens: one 16-token tile (by_tile) or all of slot blockIdx.y
  GridTile gt;
  if (!grid_row(args.seg, args.ranks, by_tile, later_rows, lane, gt)) return;
  const int s = gt.slot;
  const int64_t t_begin = gt.begin, t_end = gt.end;
  const int rank = gt.rank;
  const int N = args.N, R = args.R;
  const int col0 = blockIdx.x * kGridCols + warp * 64;
  if (t_end <= t_begin || rank <= 0 || col0 >= N) return;  // no barrier follows
  const float scale = __ldg(args.scales + s);
  const int kr = min(rank, R);
  const int rr = min(RP, (kr + 15) & ~15);  // rows of B that meet a non-zero tmp column

  const uint32_t stage = smem_u32(smem + warp * Cfg::kStageBytes);
  const uint32_t regroup = smem_u32(smem + kGridWarps * Cfg::kStageBytes + warp * Cfg::kRegroupBytes);
  // B[s, 0:rr, col0:col0 + 64]: row k (128 bytes) with 16-byte chunk j at j ^ (k & 7)
  {
    const uint8_t* src = args.b + ((int64_t)s * R * N + col0) * 2;
    for (int q = lane; q < rr * 8; q += 32) {
      const int k = q >> 3, j = q & 7;
      cp_async16(stage + k * 128 + ((j ^ (k & 7)) << 4), src + ((int64_t)k * N + j * 8) * 2);
    }
    cp_async_commit();
  }
  const int g = lane >> 2;  // fragment row group
  const int t = lane & 3;   // lane within the quad
  const int m = lane >> 3;  // ldmatrix matrix of this lane
  // stmatrix: lane l writes row l & 7 of matrix l >> 3; ld: row g, columns 8t .. (64-byte rows,
  // 16-byte chunk j of row r at j ^ ((r >> 1) & 3))
  const uint32_t rg_st = regroup + (lane & 7) * 64 + 16 * ((lane >> 3) ^ (((lane & 7) >> 1) & 3));
  const uint32_t rg_ld = regroup + g * 64 + 16 * (t ^ ((g >> 1) & 3));
  bool staged = false;
  for (int64_t a = t_begin; a < t_end; a += kGridTile) {
    const int cnt = (int)min((int64_t)kGridTile, t_end - a);
    const bool v0 = g < cnt, v1 = g + 8 < cnt;  // this lane's tile rows g and g + 8
    const int64_t tok0 = v0 ? (int64_t)ld_cg_i32(args.seg.token_index + a + g) : 0;
    const int64_t tok1 = v1 ? (int64_t)ld_cg_i32(args.seg.token_index + a + g + 8) : 0;
    uint8_t* y0 = args.y + (tok0 * N + col0) * 2;
    uint8_t* y1 = args.y + (tok1 * N + col0) * 2;
    uint4 yv[2][2];
#pragma unroll
    for (int blk = 0; blk < 2; ++blk) {
      const int col = 32 * blk + 8 * t;
      yv[blk][0] = v0 ? ld_stream16(y0 + col * 2) : make_uint4(0u, 0u, 0u, 0u);
      yv[blk][1] = v1 ? ld_stream16(y1 + col * 2) : make_uint4(0u, 0u, 0u, 0u);
    }
    // tmp is the previous kernel's output (programmatic launch after the shrink)
    griddep_wait();
    uint32_t fa[RP / 16][4];  // A fragments: tmp rows, columns >= kr read as zero
    {
      const uint8_t* t0 = args.tmp + tok0 * R * 2;
      const uint8_t* t1 = args.tmp + tok1 * R * 2;
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
    if (!staged) {
      cp_async_wait_all();
      __syncwarp();
      staged = true;
    }
#pragma unroll
    for (int blk = 0; blk < 2; ++blk) {
      float acc[4][4];
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
#pragma unroll
      for (int st = 0; st < RP / 16; ++st) {
        if (16 * st < rr) {
#pragma unroll
          for (int jb = 0; jb < 4; jb += 2) {
            const int c0 = 32 * blk + 8 * (jb + (m >> 1));
            const int k = 16 * st + 8 * (m & 1) + (lane & 7);
            uint32_t bf[4];
            ldsm_x4_trans(stage + k * 128 + 16 * (((c0 >> 3) & 7) ^ (k & 7)), bf);
            mma_16816<BF16>(acc[jb], fa[st], bf[0], bf[1]);
            mma_16816<BF16>(acc[jb + 1], fa[st], bf[2], bf[3]);
          }
        }
      }
      // delta = round(scale * acc), regrouped so that each lane holds its 8 columns
      uint32_t d0[4], d1[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        d0[j] = pack2<BF16>(scale * acc[j][0], scale * acc[j][1]);
        d1[j] = pack2<BF16>(scale * acc[j][2], scale * acc[j][3]);
      }
      stsm_x4(rg_st, d0);
      stsm_x4(rg_st + 8 * 64, d1);
      __syncwarp();
      lds_v4(rg_ld, d0);
      lds_v4(rg_ld + 8 * 64, d1);
      __syncwarp();
      const int col = 32 * blk + 8 * t;
      if (v0) {
        const uint4& yv0 = yv[blk][0];
        *reinterpret_cast<uint4*>(y0 + col * 2) = make_uint4(
            add2<BF16>(yv0.x, d0[0]), add2<BF16>(yv0.y, d0[1]), add2<BF16>(yv0.z, d0[2]), add2<BF16>(yv0.w, d0[3]));
      }
      if (v1) {
        const uint4& yv1 = yv[blk][1];
        *reinterpret_cast<uint4*>(y1 + col * 2) = make_uint4(
            add2<BF16>(yv1.x, d1[0]), add2<BF16>(yv1.y, d1[1]), add2<BF16>(yv1.z, d1[2]), add2<BF16>(yv1.w, d1[3]));
      }
    }
  }
}

// ------------------------------------------------------------------- shrink
// Grid (KP, slots), clusters (KP, 1, 1); part q covers K rows
// [q * kp_rows, (q + 1) * kp_rows) (kp_rows a multiple of 32).
template <int RP, bool BF16>
__global__ void __launch_bounds__(kGridThreads, 2)
    sgmv_shrink_grid_kernel(const ShrinkArgs args, int kp_rows, bool by_tile, int later_rows) {
  using Cfg = ShrinkGridCfg<RP>;
  using E = Elem<BF16>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  griddep_wait();    // inputs (segment table, x) come from earlier kernels
  griddep_launch();  // the expand may start on SMs this grid releases
  // this cluster's tokens: one 16-token tile (by_tile) or all of slot blockIdx.y
  GridTile gt;
  if (!grid_row(args.seg, args.ranks, by_tile, later_rows, lane, gt)) return;  // uniform (one grid row)
  const int s = gt.slot;
  const int64_t t_begin = gt.begin, t_end = gt.end;
  const int rank = gt.rank;
  if (t_end <= t_begin || rank <= 0) return;  // uniform across the cluster (one slot)
  const int K = args.K, R = args.R;
  const int n_eff = min(rank * args.stack_num, R);
  const int rr = min(RP, (n_eff + 15) & ~15);  // columns of A this slot uses
  const int chunks = rr >> 3;                  // 16-byte pieces per staged row
  const int k_lo = min(K, (int)blockIdx.x * kp_rows);
  const int nbc = (min(K, k_lo + kp_rows) - k_lo) >> 5;  // 32-row blocks of this part
  const int wb0 = warp * nbc / kGridWarps, wb1 = (warp + 1) * nbc / kGridWarps;
  const uint32_t stage = smem_u32(smem + warp * Cfg::kStageBytes);
  float* cpart = reinterpret_cast<float*>(smem + kGridWarps * Cfg::kStageBytes);
  const int g = lane >> 2;  // fragment row group
  const int t = lane & 3;   // lane within the quad
  const int mi = lane >> 3;
  const uint8_t* src = args.a + ((int64_t)s * K + k_lo) * R * 2;

  for (int64_t a = t_begin; a < t_end; a += kGridTile) {
    const int cnt = (int)min((int64_t)kGridTile, t_end - a);
    float acc[RP / 16][2][4];  // D^T tiles: rank rows 16 rt .., tile tokens 8 nt ..
#pragma unroll
    for (int rt = 0; rt < RP / 16; ++rt)
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) acc[rt][nt][0] = acc[rt][nt][1] = acc[rt][nt][2] = acc[rt][nt][3] = 0.f;
    const bool v0 = g < cnt, v1 = g + 8 < cnt;
    const uint8_t* x0 = args.x + (v0 ? (int64_t)ld_cg_i32(args.seg.token_index + a + g) : 0) * K * 2;
    const uint8_t* x1 = args.x + (v1 ? (int64_t)ld_cg_i32(args.seg.token_index + a + g + 8) : 0) * K * 2;
    for (int bb = wb0; bb < wb1; bb += kGridRows / 32) {
      const int nbb = min(kGridRows / 32, wb1 - bb);
      // rows [32 bb, 32 (bb + nbb)) of the part: position 8 cc + 2 m + e of a block
      // holds row 8 m + 2 cc + e, pieces swizzled as win_offset<RP>; consecutive
      // lanes fill consecutive positions (conflict-free shared-memory writes)
      for (int q = lane; q < nbb * 32 * chunks; q += 32) {
        const int pos = q / chunks, j = q - pos * chunks;
        const int pb = pos & 31;
        const int row = (pos & ~31) + 8 * ((pb >> 1) & 3) + 2 * (pb >> 3) + (pb & 1);
        cp_async16(stage + win_offset<RP>(pos, j), src + ((int64_t)(32 * bb + row) * R + 8 * j) * 2);
      }
      cp_async_commit();
      uint4 xa[kGridRows / 32][2];
#pragma unroll
      for (int u = 0; u < kGridRows / 32; ++u) {
        const int col = k_lo + 32 * (bb + u) + 8 * t;
        const bool in = u < nbb;
        xa[u][0] = (v0 && in) ? ld_stream16(x0 + col * 2) : make_uint4(0u, 0u, 0u, 0u);
        xa[u][1] = (v1 && in) ? ld_stream16(x1 + col * 2) : make_uint4(0u, 0u, 0u, 0u);
      }
      cp_async_wait_all();
      __syncwarp();
#pragma unroll
      for (int u = 0; u < kGridRows / 32; ++u) {
        if (u < nbb) {
          // B fragments of k16 step st: tokens g (x0) and 8 + g (x1), k = 8t + 4st + {0,1} / {2,3}
          const uint32_t fb0[2][2] = {{xa[u][0].x, xa[u][0].y}, {xa[u][0].z, xa[u][0].w}};
          const uint32_t fb1[2][2] = {{xa[u][1].x, xa[u][1].y}, {xa[u][1].z, xa[u][1].w}};
#pragma unroll
          for (int st = 0; st < 2; ++st) {
            const int pos = u * 32 + (2 * st + (mi >> 1)) * 8 + (lane & 7);
#pragma unroll
            for (int rt = 0; rt < RP / 16; ++rt) {
              if (16 * rt < rr) {
                uint32_t fa[4];
                ldsm_x4_trans(stage + win_offset<RP>(pos, 2 * rt + (mi & 1)), fa);
                mma_16816<BF16>(acc[rt][0], fa, fb0[st][0], fb0[st][1]);
                mma_16816<BF16>(acc[rt][1], fa, fb1[st][0], fb1[st][1]);
              }
            }
          }
        }
      }
      __syncwarp();  // the next copies overwrite the stage
    }

    // warp partials (in the warp's own stage) -> CTA partial -> cluster sum in CTA 0
    {
      float* p = reinterpret_cast<float*>(smem + warp * Cfg::kStageBytes);  // [token][rank]
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
    // the token of the tmp row this thread writes below (one piece per thread:
    // cnt * RP / 8 <= kGridThreads), loaded before the barriers hide its latency
    static_assert(kGridTile * (RP / 8) <= kGridThreads, "one tmp piece per thread");
    const int64_t tok_w = threadIdx.x < cnt * (RP / 8) ? ld_cg_i32(args.seg.token_index + a + threadIdx.x / (RP / 8)) : 0;
    __syncthreads();
    for (int i = threadIdx.x; i < kGridTile * RP; i += kGridThreads) {
      float v = 0.f;
#pragma unroll
      for (int w = 0; w < kGridWarps; ++w) v += reinterpret_cast<const float*>(smem + w * Cfg::kStageBytes)[i];
      cpart[i] = v;
    }
    cluster_sync();
    if (cluster_ctarank() == 0) {
      const int kp = (int)gridDim.x;  // the cluster spans the K parts
      if (threadIdx.x < cnt * (RP / 8)) {
        const int row = threadIdx.x / (RP / 8), cg = threadIdx.x - row * (RP / 8);
        float v[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e] = 0.f;
        const uint32_t local = smem_u32(cpart + row * RP + cg * 8);
        for (int q = 0; q < kp; ++q) {
          const uint32_t addr = cluster_map(local, (uint32_t)q);
          const float4 lo = ld_cluster_f4(addr), hi = ld_cluster_f4(addr + 16);
          v[0] += lo.x; v[1] += lo.y; v[2] += lo.z; v[3] += lo.w;
          v[4] += hi.x; v[5] += hi.y; v[6] += hi.z; v[7] += hi.w;
        }
        uint32_t out[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int c0 = cg * 8 + 2 * e;
          out[e] = (uint32_t)E::from_f(c0 < n_eff ? v[2 * e] : 0.f) |
                   ((uint32_t)E::from_f(c0 + 1 < n_eff ? v[2 * e + 1] : 0.f) << 16);
        }
        *reinterpret_cast<uint4*>(args.tmp + (tok_w * R + cg * 8) * 2) = make_uint4(out[0], out[1], out[2], out[3]);
      }
    }
    cluster_sync();  // the parts' partials and stages are reused by the next tile
  }
}

}  // namespace plora
