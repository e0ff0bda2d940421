// Device-side segment construction: groups the active tokens of a batch by
// slot with a stable (slot, row, position) order, and the reference-compatible
// flat tile schedule.  Integer work only; results are bit-exact and
// deterministic (no atomics decide an order).
//
// The table kernels are launched programmatically: each may start while its
// predecessor in the stream finishes, waits (griddep_wait) before reading or
// writing global memory, reads what earlier kernels wrote with volatile L2
// loads (which stay below the wait), and lets its successor start at once.
//
// Replaces the host-synchronising schedule construction of the reference,
// src/polylora/sgmv.py:29-61 (_build_flat_schedule) and sgmv.py:304-309, and
// the per-row slot lookups of layers.py:124-130.
#pragma once

#include "common.cuh"

namespace plora {

constexpr int kSegRowsPerBlock = 256;  // rows counted per block (8 warps)
constexpr int kSegMaxSlots = 4096;     // slot-count limit of the segment kernels

// Workspace layout (bytes, each part 256-aligned):
//   partial[num_slots][num_blocks] int32  per-slot per-block token counts,
//                                         rewritten in place to the prefix over
//                                         earlier blocks of the same slot
//   row_off[num_rows]              int32  token offset of a row within its block+slot
//   row_info[num_rows]             int32  slot (>= 0) or -1 when inactive
__host__ __device__ inline size_t align256(size_t v) { return (v + 255) & ~(size_t)255; }

struct SegWorkspace {
  int32_t* partial;
  int32_t* row_off;
  int32_t* row_info;
};

__host__ inline size_t seg_workspace_bytes(int64_t num_rows, int32_t num_slots) {
  const int64_t blocks = (num_rows + kSegRowsPerBlock - 1) / kSegRowsPerBlock;
  return align256((size_t)blocks * (size_t)num_slots * 4) + 2 * align256((size_t)num_rows * 4);
}

__host__ inline SegWorkspace seg_workspace_carve(void* ws, int64_t num_rows, int32_t num_slots) {
  const int64_t blocks = (num_rows + kSegRowsPerBlock - 1) / kSegRowsPerBlock;
  char* p = static_cast<char*>(ws);
  SegWorkspace w;
  w.partial = reinterpret_cast<int32_t*>(p);
  p += align256((size_t)blocks * (size_t)num_slots * 4);
  w.row_off = reinterpret_cast<int32_t*>(p);
  p += align256((size_t)num_rows * 4);
  w.row_info = reinterpret_cast<int32_t*>(p);
  return w;
}

// Pass 1: per block of 256 rows, the token count of every slot and, for each
// active row, the offset of its tokens among the block's rows of that slot in
// row order.  Warps take turns (8 steps); inside a warp the same-slot prefix
// comes from __match_any_sync groups and a shuffle scan.
__global__ void __launch_bounds__(kSegRowsPerBlock) seg_count_kernel(
    const int64_t* __restrict__ weight_indices, const int32_t* __restrict__ seq_lens,
    const int32_t* __restrict__ lora_ranks, int64_t num_rows, int64_t max_seq, int32_t num_slots,
    SegWorkspace ws) {
  extern __shared__ int32_t cnt[];  // [num_slots]
  for (int s = threadIdx.x; s < num_slots; s += blockDim.x) cnt[s] = 0;
  griddep_wait();
  griddep_launch();

  const int64_t row = (int64_t)blockIdx.x * kSegRowsPerBlock + threadIdx.x;
  int key = -1;
  int len = 0;
  if (row < num_rows) {
    const int64_t slot = ld_cg_i64(weight_indices + row);
    int64_t l = ld_cg_i32(seq_lens + row);  // issued beside the slot's load
    if (slot < 0 || slot >= num_slots) {
      raise_status(PLORA_DEV_SLOT_RANGE);
    } else {
      const int32_t rank = ld_cg_i32(lora_ranks + slot);
      l = l < 0 ? 0 : (l > max_seq ? max_seq : l);
      if (rank > 0 && l > 0) {
        key = (int)slot;
        len = (int)l;
      }
    }
  }
  __syncthreads();

  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const unsigned peers = __match_any_sync(0xffffffffu, key);
  // Exclusive prefix of len over lower lanes of the same group.
  int prefix = 0;
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const int lj = __shfl_sync(0xffffffffu, len, j);
    if (j < lane && ((peers >> j) & 1u)) prefix += lj;
  }
  const bool group_last = (31 - __clz(peers)) == lane;

  for (int w = 0; w < kSegRowsPerBlock / 32; ++w) {
    if (warp == w && key >= 0) {
      const int base = cnt[key];
      if (row < num_rows) ws.row_off[row] = base + prefix;
      __syncwarp(peers);
      if (group_last) cnt[key] = base + prefix + len;
    }
    __syncthreads();
  }
  if (row < num_rows) ws.row_info[row] = key;
  for (int s = threadIdx.x; s < num_slots; s += blockDim.x)
    ws.partial[(int64_t)s * gridDim.x + blockIdx.x] = cnt[s];
}

// Pass 2 (one block of 1024): per slot (one warp each, lanes over blocks),
// partial[s][b] becomes the prefix over blocks b' < b; then slot_start is the
// exclusive scan over slots of the per-slot totals.
__global__ void __launch_bounds__(1024) seg_scan_kernel(int32_t num_blocks, int32_t num_slots,
                                                         SegWorkspace ws,
                                                         int32_t* __restrict__ slot_start) {
  extern __shared__ int32_t totals[];  // [num_slots]
  __shared__ int32_t warp_sums[32];
  __shared__ int32_t carry;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int nwarps = blockDim.x >> 5;
  griddep_wait();
  griddep_launch();
  for (int s = warp; s < num_slots; s += nwarps) {
    int32_t* row = ws.partial + (int64_t)s * num_blocks;
    int run = 0;
    for (int b0 = 0; b0 < num_blocks; b0 += 32) {
      const int b = b0 + lane;
      const int v = b < num_blocks ? ld_cg_i32(row + b) : 0;
      int incl = v;
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        const int u = __shfl_up_sync(0xffffffffu, incl, d);
        if (lane >= d) incl += u;
      }
      if (b < num_blocks) row[b] = run + incl - v;
      run += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) totals[s] = run;
  }
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  for (int s0 = 0; s0 < num_slots; s0 += blockDim.x) {
    const int s = s0 + threadIdx.x;
    const int total = s < num_slots ? totals[s] : 0;
    int incl = total;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, d);
      if (lane >= d) incl += v;
    }
    if (lane == 31) warp_sums[warp] = incl;
    __syncthreads();
    if (warp == 0) {
      int v = (lane < nwarps) ? warp_sums[lane] : 0;
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        const int u = __shfl_up_sync(0xffffffffu, v, d);
        if (lane >= d) v += u;
      }
      warp_sums[lane] = v;  // inclusive over warps
    }
    __syncthreads();
    const int excl = carry + (warp > 0 ? warp_sums[warp - 1] : 0) + incl - total;
    if (s < num_slots) slot_start[s] = excl;
    __syncthreads();
    if (threadIdx.x == blockDim.x - 1) carry = excl + total;
    __syncthreads();
  }
  if (threadIdx.x == 0) slot_start[num_slots] = carry;
}

// Pass 3: one warp per row writes the row's token ids at its final position
// slot_start[slot] + prefix of earlier blocks + offset within the block.
__global__ void __launch_bounds__(256) seg_place_kernel(int64_t num_rows, int64_t max_seq,
                                                         const int32_t* __restrict__ seq_lens,
                                                         int32_t num_blocks, SegWorkspace ws,
                                                         const int32_t* __restrict__ slot_start,
                                                         int32_t* __restrict__ token_index) {
  griddep_wait();
  griddep_launch();
  const int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= num_rows) return;
  const int key = ld_cg_i32(ws.row_info + row);
  if (key < 0) return;
  int64_t l = ld_cg_i32(seq_lens + row);
  l = l < 0 ? 0 : (l > max_seq ? max_seq : l);
  const int64_t blk = row / kSegRowsPerBlock;
  const int64_t dst = (int64_t)ld_cg_i32(slot_start + key) + ld_cg_i32(ws.partial + (int64_t)key * num_blocks + blk) +
                      ld_cg_i32(ws.row_off + row);
  const int64_t tok0 = row * max_seq;
  for (int64_t m = lane; m < l; m += 32) token_index[dst + m] = (int32_t)(tok0 + m);
}

// Passes 2 and 3 in one launch, for tables whose count matrix (num_slots x
// count blocks) fits shared memory: every block loads the whole matrix (it is
// in L2), turns each slot's counts into the prefix over count blocks and the
// slot totals into slot_start (block 0 writes it out), then places its own
// contiguous range of rows, one warp per row.  The scan is repeated in every
// block; it costs a few microseconds of SM time and saves a launch and a
// round trip through global memory.  1024 threads.
constexpr int kSegScanPlaceMaxInts = 12288;  // count-matrix limit: 48 KB of shared memory

__global__ void __launch_bounds__(1024) seg_scan_place_kernel(
    int64_t num_rows, int64_t max_seq, const int32_t* __restrict__ seq_lens, int32_t num_blocks,
    int32_t num_slots, SegWorkspace ws, int32_t* __restrict__ slot_start, int32_t* __restrict__ token_index) {
  extern __shared__ int32_t sm[];
  int32_t* part = sm;                                        // [num_slots][num_blocks]
  int32_t* base = sm + (int64_t)num_slots * num_blocks;      // [num_slots + 1] slot starts
  __shared__ int32_t warp_sums[32];
  __shared__ int32_t carry;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int nwarps = blockDim.x >> 5;
  griddep_wait();
  griddep_launch();
  const int n = num_slots * num_blocks;
  for (int i = threadIdx.x; i < n; i += blockDim.x) part[i] = ld_cg_i32(ws.partial + i);
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  // per slot (a warp each): counts -> prefix over count blocks; the total into base[s]
  for (int s = warp; s < num_slots; s += nwarps) {
    int32_t* row = part + (int64_t)s * num_blocks;
    int run = 0;
    for (int b0 = 0; b0 < num_blocks; b0 += 32) {
      const int b = b0 + lane;
      const int v = b < num_blocks ? row[b] : 0;
      int incl = v;
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        const int u = __shfl_up_sync(0xffffffffu, incl, d);
        if (lane >= d) incl += u;
      }
      if (b < num_blocks) row[b] = run + incl - v;
      run += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) base[s] = run;
  }
  __syncthreads();
  // exclusive scan of the totals over slots, in place
  for (int s0 = 0; s0 < num_slots; s0 += blockDim.x) {
    const int s = s0 + threadIdx.x;
    const int total = s < num_slots ? base[s] : 0;
    int incl = total;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, d);
      if (lane >= d) incl += v;
    }
    if (lane == 31) warp_sums[warp] = incl;
    __syncthreads();
    if (warp == 0) {
      int v = (lane < nwarps) ? warp_sums[lane] : 0;
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        const int u = __shfl_up_sync(0xffffffffu, v, d);
        if (lane >= d) v += u;
      }
      warp_sums[lane] = v;
    }
    __syncthreads();
    const int excl = carry + (warp > 0 ? warp_sums[warp - 1] : 0) + incl - total;
    __syncthreads();  // every thread has read base[] of this chunk and carry
    if (s < num_slots) base[s] = excl;
    if (threadIdx.x == blockDim.x - 1) carry = excl + total;
    __syncthreads();
  }
  if (threadIdx.x == 0) base[num_slots] = carry;
  __syncthreads();
  if (blockIdx.x == 0)
    for (int s = threadIdx.x; s <= num_slots; s += blockDim.x) slot_start[s] = base[s];
  // this block's rows, 1024 at a time: a thread loads one row's metadata (all
  // rows' loads in flight together), then one warp per row writes its ids
  __shared__ int32_t row_dst[1024], row_len[1024];
  const int64_t r0 = num_rows * blockIdx.x / gridDim.x, r1 = num_rows * (blockIdx.x + 1) / gridDim.x;
  for (int64_t c = r0; c < r1; c += blockDim.x) {
    const int64_t row = c + threadIdx.x;
    int32_t dst = -1, len = 0;
    if (row < r1) {
      const int key = ld_cg_i32(ws.row_info + row);
      const int32_t off = ld_cg_i32(ws.row_off + row);
      int64_t l = ld_cg_i32(seq_lens + row);
      if (key >= 0) {
        dst = base[key] + part[(int64_t)key * num_blocks + row / kSegRowsPerBlock] + off;
        len = (int32_t)(l < 0 ? 0 : (l > max_seq ? max_seq : l));
      }
    }
    row_dst[threadIdx.x] = dst;
    row_len[threadIdx.x] = len;
    __syncthreads();
    const int n = (int)(r1 - c < (int64_t)blockDim.x ? r1 - c : (int64_t)blockDim.x);
    for (int i = warp; i < n; i += nwarps) {
      if (row_dst[i] < 0) continue;
      const int64_t tok0 = (c + i) * max_seq;
      for (int m = lane; m < row_len[i]; m += 32) token_index[row_dst[i] + m] = (int32_t)(tok0 + m);
    }
    __syncthreads();
  }
}

// One-launch builder for small batches (decode steps): one block of 1024
// threads, one thread per row, the same table as the three passes above.
//   1. key / len per row exactly as seg_count_kernel;
//   2. per warp, the same-slot prefix of lower lanes (__match_any_sync group +
//      shuffle scan); the group's last lane writes the warp's token count of
//      that slot into cnt[warp][slot] (one group per slot per warp: no races);
//   3. per slot (thread s), cnt[.][s] becomes the exclusive prefix over warps,
//      i.e. over lower rows, and the slot total goes into a block scan over
//      slots that gives slot_start;
//   4. a row's first position is slot_start[slot] + cnt[warp][slot] + prefix;
//      one warp per row then writes the row's token ids.
// Rows <= kSegSmallRows, slots <= kSegSmallSlots and tokens <= kSegSmallTokens
// (a single SM writes every token id).  Needs no workspace.
constexpr int kSegSmallRows = 1024;
constexpr int kSegSmallSlots = 256;
constexpr int64_t kSegSmallTokens = 16384;

__global__ void __launch_bounds__(1024) seg_small_kernel(
    const int64_t* __restrict__ weight_indices, const int32_t* __restrict__ seq_lens,
    const int32_t* __restrict__ lora_ranks, int32_t num_rows, int64_t max_seq, int32_t num_slots,
    int32_t* __restrict__ slot_start, int32_t* __restrict__ token_index) {
  __shared__ int32_t cnt[32][kSegSmallSlots];  // per-warp per-slot counts, then offsets
  __shared__ int32_t start[kSegSmallSlots];
  __shared__ int32_t row_dst[kSegSmallRows];   // first token position of a row, -1 when inactive
  __shared__ int32_t warp_sums[32];
  const int t = threadIdx.x;
  const int lane = t & 31;
  const int warp = t >> 5;
  for (int i = t; i < 32 * kSegSmallSlots; i += blockDim.x) (&cnt[0][0])[i] = 0;
  griddep_wait();
  griddep_launch();

  int key = -1;
  int len = 0;
  if (t < num_rows) {
    const int64_t slot = ld_cg_i64(weight_indices + t);
    if (slot < 0 || slot >= num_slots) {
      raise_status(PLORA_DEV_SLOT_RANGE);
    } else {
      const int32_t rank = ld_cg_i32(lora_ranks + slot);
      int64_t l = ld_cg_i32(seq_lens + t);
      l = l < 0 ? 0 : (l > max_seq ? max_seq : l);
      if (rank > 0 && l > 0) {
        key = (int)slot;
        len = (int)l;
      }
    }
  }
  const unsigned peers = __match_any_sync(0xffffffffu, key);
  int prefix = 0;
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const int lj = __shfl_sync(0xffffffffu, len, j);
    if (j < lane && ((peers >> j) & 1u)) prefix += lj;
  }
  const bool group_last = (31 - __clz(peers)) == lane;
  __syncthreads();  // cnt zeroed
  if (key >= 0 && group_last) cnt[warp][key] = prefix + len;
  __syncthreads();

  int total = 0;
  if (t < num_slots) {
#pragma unroll 8
    for (int w = 0; w < 32; ++w) {
      const int v = cnt[w][t];
      cnt[w][t] = total;
      total += v;
    }
  }
  int incl = total;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const int u = __shfl_up_sync(0xffffffffu, incl, d);
    if (lane >= d) incl += u;
  }
  if (lane == 31) warp_sums[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int v = warp_sums[lane];
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int u = __shfl_up_sync(0xffffffffu, v, d);
      if (lane >= d) v += u;
    }
    warp_sums[lane] = v;  // inclusive over warps
  }
  __syncthreads();
  if (t < num_slots) {
    const int excl = (warp > 0 ? warp_sums[warp - 1] : 0) + incl - total;
    start[t] = excl;
    slot_start[t] = excl;
  }
  if (t == 0) slot_start[num_slots] = warp_sums[31];
  __syncthreads();
  if (t < num_rows) row_dst[t] = key >= 0 ? start[key] + cnt[warp][key] + prefix : -1;
  __syncthreads();

  for (int r = warp; r < num_rows; r += 32) {
    const int dst = row_dst[r];
    if (dst < 0) continue;
    int64_t l = ld_cg_i32(seq_lens + r);
    l = l < 0 ? 0 : (l > max_seq ? max_seq : l);
    const int64_t tok0 = (int64_t)r * max_seq;
    for (int64_t m = lane; m < l; m += 32) token_index[dst + m] = (int32_t)(tok0 + m);
  }
}

// Flat tile schedule of the reference (sgmv.py:29-61), one block with carry:
//   num_n_tiles[b] = cdiv(n_eff[b], block_n)
//   tiles[b]       = (seq_len == 0 || n_eff == 0) ? 0 : cdiv(seq_len, block_m) * num_n_tiles[b]
//   cum_tiles      = [0, cumsum(tiles)]
__global__ void __launch_bounds__(1024) flat_schedule_kernel(const int32_t* __restrict__ seq_lens,
                                                              const int32_t* __restrict__ n_eff,
                                                              int64_t num_rows, int32_t block_m,
                                                              int32_t block_n,
                                                              int32_t* __restrict__ cum_tiles,
                                                              int32_t* __restrict__ num_n_tiles) {
  __shared__ int32_t warp_sums[32];
  __shared__ int32_t carry;
  if (threadIdx.x == 0) {
    carry = 0;
    cum_tiles[0] = 0;
  }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  for (int64_t b0 = 0; b0 < num_rows; b0 += blockDim.x) {
    const int64_t b = b0 + threadIdx.x;
    int32_t tiles = 0;
    if (b < num_rows) {
      const int32_t sl = seq_lens[b];
      const int32_t ne = n_eff[b];
      const int32_t nm = (sl + block_m - 1) / block_m;
      const int32_t nn = (ne + block_n - 1) / block_n;
      num_n_tiles[b] = nn;
      tiles = (sl == 0 || ne == 0) ? 0 : nm * nn;
    }
    int32_t incl = tiles;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int32_t v = __shfl_up_sync(0xffffffffu, incl, d);
      if (lane >= d) incl += v;
    }
    if (lane == 31) warp_sums[warp] = incl;
    __syncthreads();
    if (warp == 0) {
      int32_t v = (lane < (int)(blockDim.x >> 5)) ? warp_sums[lane] : 0;
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        const int32_t u = __shfl_up_sync(0xffffffffu, v, d);
        if (lane >= d) v += u;
      }
      warp_sums[lane] = v;
    }
    __syncthreads();
    const int32_t incl_all = carry + (warp > 0 ? warp_sums[warp - 1] : 0) + incl;
    if (b < num_rows) cum_tiles[b + 1] = incl_all;
    __syncthreads();
    if (threadIdx.x == blockDim.x - 1) carry = incl_all;
    __syncthreads();
  }
}

// Right-padding check of an attention mask (rows x width, contiguous, elements
// of elem_bytes bytes): row r must be non-zero exactly at positions <
// seq_lens[r], seq_lens being the row sums the caller computed from the same
// mask.  A float mask (is_float) ignores the sign bit, so -0.0 counts as zero
// as bool() has it.  A violation ORs PLORA_DEV_PADDING into the device status
// word; nothing is read back.  One block per row.
// Reference: src/polylora/context.py:37-45 (assert_right_padded).
__global__ void mask_padding_kernel(const uint8_t* __restrict__ mask, int elem_bytes, int is_float,
                                    const int64_t* __restrict__ seq_lens, int64_t width) {
  const int64_t r = blockIdx.x;
  const int64_t len = seq_lens[r];
  const uint8_t* row = mask + r * width * elem_bytes;
  const uint64_t value_bits = !is_float ? ~0ull : (~0ull >> (65 - 8 * elem_bytes));  // drop the sign bit
  bool bad = false;
  for (int64_t p = threadIdx.x; p < width; p += blockDim.x) {
    uint64_t v;
    switch (elem_bytes) {
      case 1: v = row[p]; break;
      case 2: v = reinterpret_cast<const uint16_t*>(row)[p]; break;
      case 4: v = reinterpret_cast<const uint32_t*>(row)[p]; break;
      default: v = reinterpret_cast<const uint64_t*>(row)[p]; break;
    }
    bad |= ((v & value_bits) != 0) != (p < len);
  }
  if (__syncthreads_or(bad) && threadIdx.x == 0) raise_status(PLORA_DEV_PADDING);
}

}  // namespace plora
