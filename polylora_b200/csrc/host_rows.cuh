// Token rows between mapped host memory and the device, for the tokens of a
// segment table only.
//
// A host-buffer caller of the LoRA op (the base output updated in place, as
// the reference's expand updates y in place: src/polylora/sgmv.py:278-328)
// needs on the device only the rows the op reads and writes: x and the base
// output of the tokens the segment table lists.  The other rows keep their
// values in host memory.  These kernels read those rows from page-locked,
// mapped host memory over PCIe straight into their places in a device buffer
// (gather), and write them back (scatter), so the bus carries the active rows
// only.  One warp moves one row at a time in 16-byte pieces, four pieces in
// flight per lane; the grid (two CTAs of 8 warps per SM) keeps several MB of
// requests in flight, which the bus needs at its latency.
//
// The launches are plain (their inputs typically come from another stream);
// griddepcontrol.wait keeps the kernel correct behind a programmatic
// predecessor too.  A token id outside [0, num_tokens) is skipped and raises
// PLORA_DEV_TOKEN_RANGE.
#pragma once

#include "common.cuh"

namespace plora {

constexpr int kRowsThreads = 256;
constexpr int kRowsUnroll = 4;  // 16-byte pieces a lane has in flight

// Copies row t (row_bytes, a multiple of 16) of src to row t of dst for every
// token t the table lists; src and dst are device-accessible addresses (one of
// them mapped host memory).
__global__ void __launch_bounds__(kRowsThreads) token_rows_copy_kernel(const uint8_t* __restrict__ src,
                                                                       uint8_t* __restrict__ dst, int64_t row_bytes,
                                                                       int64_t num_tokens,
                                                                       const int32_t* __restrict__ slot_start,
                                                                       const int32_t* __restrict__ token_index,
                                                                       int32_t num_slots) {
  griddep_wait();  // the table comes from the kernels before this one
  griddep_launch();
  const int lane = threadIdx.x & 31;
  const int64_t warp = ((int64_t)blockIdx.x * kRowsThreads + threadIdx.x) >> 5;
  const int64_t warps = ((int64_t)gridDim.x * kRowsThreads) >> 5;
  const int64_t n = ld_cg_i32(slot_start + num_slots);  // tokens in the table
  const int64_t pieces = row_bytes >> 4;
  for (int64_t i = warp; i < n; i += warps) {
    const int64_t t = ld_cg_i32(token_index + i);
    if (t < 0 || t >= num_tokens) {  // uniform across the warp
      if (lane == 0) raise_status(PLORA_DEV_TOKEN_RANGE);
      continue;
    }
    const uint4* s = reinterpret_cast<const uint4*>(src + t * row_bytes);
    uint4* d = reinterpret_cast<uint4*>(dst + t * row_bytes);
    for (int64_t p0 = lane; p0 < pieces; p0 += 32 * kRowsUnroll) {
      uint4 v[kRowsUnroll];
#pragma unroll
      for (int u = 0; u < kRowsUnroll; ++u) {
        const int64_t p = p0 + 32 * u;
        if (p < pieces) v[u] = s[p];
      }
#pragma unroll
      for (int u = 0; u < kRowsUnroll; ++u) {
        const int64_t p = p0 + 32 * u;
        if (p < pieces) d[p] = v[u];
      }
    }
  }
}

}  // namespace plora
