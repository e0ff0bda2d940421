// C ABI of libpolylora_b200.so: argument checks, TMA tensor maps, launch
// configuration and dispatch between the tensor-core (bf16/fp16) and CUDA-core
// kernels.  One translation unit so the device status word is shared.
#include <cudaTypedefs.h>

#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "common.cuh"
#include "segments.cuh"
#include "sgmv_simt.cuh"
#include "sgmv_grid.cuh"
#include "host_rows.cuh"
#include "sgmv_stream.cuh"
#include "peft_pack.h"

using namespace plora;

// Scratch of plora_sgmv_a_fwd_noalloc: segment scratch + slot table for one
// batch, resident on every device that loads the library.  Host code must not
// use this symbol as a pointer; it is a host-side stand-in for the device
// array, whose address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_noalloc_scratch[PLORA_NOALLOC_SCRATCH_BYTES];

namespace {

thread_local std::string g_last_error;

int fail(int status, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return status;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(PLORA_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

#define PLORA_CUDA(call, what)             \
  do {                                     \
    cudaError_t _e = (call);               \
    if (_e != cudaSuccess) return cuda_fail(_e, what); \
  } while (0)

constexpr int kMaxDevices = 64;

// Shared-memory bytes of the per-slot table staged by the token-split kernels.
size_t tab_bytes(int32_t ns) { return (size_t)slot_tab_bytes(ns); }

struct DeviceInfo {
  int sm_count = 0;
  bool attrs_set = false;
};
DeviceInfo g_dev[kMaxDevices];
std::mutex g_dev_mu;

// Batches of at most this many tokens per SM run the slot-grid kernels
// (sgmv_grid.cuh): their slots have few tokens each, so giving every (slot,
// weight part) a CTA beats giving each CTA a share of the tokens (which makes
// every CTA stream the whole LoRA weights of each slot it touches).
std::atomic<int64_t> g_wsplit_tokens_per_sm{16};

// Rank-16 calls of many tokens run the stream kernels (sgmv_stream.cuh) when
// this is non-zero; 0 keeps them on the windowed mma kernels.  2 (the default)
// also runs plora_sgmv_shrink_expand as the fused stream kernel, 1 as the two.
std::atomic<int32_t> g_stream_kernels{2};

// A CTA's share of the token list must fit the stream kernels' shared-memory
// copy of its token ids.  Shares are cost-balanced (stream_share): one holds at
// most ceil((tokens + slot_cost * active slots) / SMs) + 1 tokens.
bool stream_share_ok(int64_t num_tokens, int64_t num_slots, int64_t slot_cost, const DeviceInfo* di) {
  const int64_t virt = num_tokens + slot_cost * num_slots;
  return (virt + di->sm_count - 1) / di->sm_count + 1 <= kStreamMaxShare;
}
bool stream_shrink_ok(int64_t R, int64_t K, int64_t num_tokens, int64_t num_slots, const DeviceInfo* di) {
  return g_stream_kernels.load(std::memory_order_relaxed) != 0 && R == kStreamRank && K % 512 == 0 &&
         K <= kStreamMaxDim && stream_share_ok(num_tokens, num_slots, kShrinkSlotCost, di);
}
bool stream_expand_ok(int64_t R, int64_t N, int64_t num_tokens, int64_t num_slots, const DeviceInfo* di) {
  return g_stream_kernels.load(std::memory_order_relaxed) != 0 && R == kStreamRank && N % 512 == 0 &&
         N <= kStreamMaxDim && stream_share_ok(num_tokens, num_slots, 0, di);  // equal token shares
}

bool use_weight_split(int64_t num_tokens, const DeviceInfo* di) {
  return num_tokens <= g_wsplit_tokens_per_sm.load(std::memory_order_relaxed) * di->sm_count;
}

int device_info(DeviceInfo** out) {
  int dev = 0;
  PLORA_CUDA(cudaGetDevice(&dev), "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(PLORA_ERR_UNSUPPORTED, "device ordinal %d", dev);
  std::lock_guard<std::mutex> lk(g_dev_mu);
  DeviceInfo& d = g_dev[dev];
  if (!d.attrs_set) {
    PLORA_CUDA(cudaDeviceGetAttribute(&d.sm_count, cudaDevAttrMultiProcessorCount, dev),
               "cudaDeviceGetAttribute");
    int major = 0, minor = 0;
    PLORA_CUDA(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev), "cc");
    PLORA_CUDA(cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev), "cc");
    if (major != 10 || minor != 0)
      return fail(PLORA_ERR_UNSUPPORTED, "device %d is sm_%d%d; this build targets sm_100a", dev,
                  major, minor);
#define SET_SMEM(kern, bytes)                                                                  \
  PLORA_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,           \
                                  (int)((bytes) + tab_bytes(kFastPathMaxSlots))),              \
             #kern);
#define SET_SMEM_BOTH(name, RPV, bytes)   \
  SET_SMEM((name<RPV, true>), bytes)      \
  SET_SMEM((name<RPV, false>), bytes)
    SET_SMEM_BOTH(sgmv_shrink_mma_kernel, 16, ShrinkMmaCfg<16>::kSmemBytes)
    SET_SMEM_BOTH(sgmv_shrink_mma_kernel, 32, ShrinkMmaCfg<32>::kSmemBytes)
    SET_SMEM_BOTH(sgmv_shrink_mma_kernel, 64, ShrinkMmaCfg<64>::kSmemBytes)
    SET_SMEM_BOTH(sgmv_expand_mma_kernel, 16, ExpandMmaCfg<16>::kSmemBytes)
    SET_SMEM_BOTH(sgmv_expand_mma_kernel, 32, ExpandMmaCfg<32>::kSmemBytes)
    SET_SMEM_BOTH(sgmv_expand_mma_kernel, 64, ExpandMmaCfg<64>::kSmemBytes)
#undef SET_SMEM_BOTH
#undef SET_SMEM
#define SET_GRID(kern, bytes)                                                                  \
  PLORA_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,           \
                                  (int)(bytes)),                                               \
             #kern);
#define SET_GRID_ALL(RPV)                                                                      \
  SET_GRID((sgmv_expand_grid_kernel<RPV, true>), ExpandGridCfg<RPV>::kSmemBytes)               \
  SET_GRID((sgmv_expand_grid_kernel<RPV, false>), ExpandGridCfg<RPV>::kSmemBytes)              \
  SET_GRID((sgmv_shrink_grid_kernel<RPV, true>), ShrinkGridCfg<RPV>::kSmemBytes)               \
  SET_GRID((sgmv_shrink_grid_kernel<RPV, false>), ShrinkGridCfg<RPV>::kSmemBytes)              \
  PLORA_CUDA(cudaFuncSetAttribute((sgmv_shrink_grid_kernel<RPV, true>),                        \
                                  cudaFuncAttributeNonPortableClusterSizeAllowed, 1), "cluster"); \
  PLORA_CUDA(cudaFuncSetAttribute((sgmv_shrink_grid_kernel<RPV, false>),                       \
                                  cudaFuncAttributeNonPortableClusterSizeAllowed, 1), "cluster");
    SET_GRID_ALL(16)
    SET_GRID_ALL(32)
    SET_GRID_ALL(64)
#undef SET_GRID_ALL
    SET_GRID((sgmv_shrink_stream_kernel<true, false>), kStreamSmemLimit)
    SET_GRID((sgmv_shrink_stream_kernel<false, false>), kStreamSmemLimit)
    SET_GRID((sgmv_shrink_stream_kernel<true, true>), kStreamSmemLimit)
    SET_GRID((sgmv_shrink_stream_kernel<false, true>), kStreamSmemLimit)
    SET_GRID((sgmv_expand_stream_kernel<true>), kStreamSmemLimit)
    SET_GRID((sgmv_expand_stream_kernel<false>), kStreamSmemLimit)
    SET_GRID(seg_scan_place_kernel, (kSegScanPlaceMaxInts + kSegMaxSlots + 1) * 4)
#undef SET_GRID
    // the row copies use no shared memory; an SM running them keeps its largest
    // shared-memory carveout, so the segment-table kernels of the next rows of
    // a host pipeline fit beside them instead of waiting for the SM to drain
    PLORA_CUDA(cudaFuncSetAttribute(token_rows_copy_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                                    (int)cudaSharedmemCarveoutMaxShared),
               "cudaFuncSetAttribute(carveout)");
    d.attrs_set = true;
  }
  *out = &d;
  return PLORA_OK;
}

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// LoRA-A (num_slots, K, R) viewed as 5-D (R, e:2, m:4, cc:4, block) with
// row k = 32 block + 8 m + 2 cc + e, so that a box lands each 32-row block
// in (cc, m, e) order: shared-memory row position 8 cc + 2 m + e.  Slots are
// folded into the block index (K % 32 == 0); the box covers `blocks` blocks.
int make_map_lora_a_blocks(CUtensorMap* map, const void* base, int dtype, uint64_t R, uint64_t K,
                           uint64_t num_slots, uint32_t blocks, CUtensorMapSwizzle swz) {
  auto enc = tensor_map_encoder();
  if (!enc) return fail(PLORA_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  const uint64_t row = R * 2;
  const cuuint64_t dims[5] = {R, 2, 4, 4, num_slots * (K / 32)};
  const cuuint64_t strides[4] = {row, 8 * row, 2 * row, 32 * row};
  const cuuint32_t box[5] = {(cuuint32_t)R, 2, 4, 4, blocks};
  const cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  const CUtensorMapDataType dt = dtype == PLORA_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                           : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUresult r = enc(map, dt, 5, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(PLORA_ERR_CUDA, "cuTensorMapEncodeTiled (LoRA-A blocks) failed (%d)", (int)r);
  return PLORA_OK;
}

// LoRA-B (num_slots, R, N) viewed as 4-D (64 columns, R, N / 64 chunks, slot):
// a box lands `chunks` 64-column chunks of all R rows, chunk-major, each chunk
// R rows of 128 bytes with the 128-byte swizzle.  Requires N % 64 == 0.
int make_map_lora_b_chunks(CUtensorMap* map, const void* base, int dtype, uint64_t R, uint64_t N,
                           uint64_t num_slots, uint32_t chunks) {
  auto enc = tensor_map_encoder();
  if (!enc) return fail(PLORA_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  const cuuint64_t dims[4] = {64, R, N / 64, num_slots};
  const cuuint64_t strides[3] = {N * 2, 128, R * N * 2};
  const cuuint32_t box[4] = {64, (cuuint32_t)R, chunks, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUtensorMapDataType dt = dtype == PLORA_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                           : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUresult r = enc(map, dt, 4, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(PLORA_ERR_CUDA, "cuTensorMapEncodeTiled (LoRA-B chunks) failed (%d)", (int)r);
  return PLORA_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

size_t elem_size(int dtype) { return dtype == PLORA_DTYPE_F32 ? 4 : 2; }

bool valid_dtype(int dtype) {
  return dtype == PLORA_DTYPE_F32 || dtype == PLORA_DTYPE_F16 || dtype == PLORA_DTYPE_BF16;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, what);
  return PLORA_OK;
}

// Workspace of the *_fwd entry points: segment scratch, slot_start, token_index.
struct FwdWorkspace {
  SegWorkspace seg;
  int32_t* slot_start;
  int32_t* token_index;
};

// num_rows x max_seq token ids fit in int32 (checked before any product is formed).
bool token_count_ok(int64_t num_rows, int64_t max_seq) {
  if (num_rows < 0 || max_seq < 0) return false;
  return max_seq == 0 || num_rows <= (int64_t)INT32_MAX / max_seq;
}

size_t fwd_workspace_bytes(int64_t num_rows, int64_t max_seq, int32_t num_slots) {
  return seg_workspace_bytes(num_rows, num_slots) + align256((size_t)(num_slots + 1) * 4) +
         align256((size_t)(num_rows * max_seq) * 4);
}

// Launches `kernel` with programmatic stream serialisation when `pdl` is set:
// the kernel may then start while its predecessor in the stream finishes and
// must call griddep_wait() before reading anything that predecessor writes.
// With cluster_x > 0 the grid is launched as clusters of cluster_x CTAs along x.
template <typename... KArgs, typename... Args>
cudaError_t launch_kernel(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                          cudaStream_t stream, bool pdl, int cluster_x, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  int n = 0;
  if (pdl) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  if (cluster_x > 0) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = (unsigned)cluster_x;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

int build_segments(const int64_t* wi, const int32_t* seq_lens, const int32_t* ranks,
                   int64_t num_rows, int64_t max_seq, int32_t num_slots, int32_t* slot_start,
                   int32_t* token_index, void* ws, size_t ws_bytes, cudaStream_t stream) {
  if (num_slots < 1 || num_slots > kSegMaxSlots)
    return fail(PLORA_ERR_UNSUPPORTED, "num_slots %d outside [1, %d]", num_slots, kSegMaxSlots);
  if (num_rows < 0 || max_seq < 0)
    return fail(PLORA_ERR_INVALID_ARGUMENT, "negative num_rows/max_seq");
  if (!token_count_ok(num_rows, max_seq))
    return fail(PLORA_ERR_UNSUPPORTED, "num_rows*max_seq exceeds int32 token ids");
  if (!slot_start) return fail(PLORA_ERR_INVALID_ARGUMENT, "slot_start is null");
  if (num_rows == 0 || max_seq == 0) {
    PLORA_CUDA(cudaMemsetAsync(slot_start, 0, (size_t)(num_slots + 1) * 4, stream), "memset");
    return PLORA_OK;
  }
  if (!wi || !seq_lens || !ranks || !token_index)
    return fail(PLORA_ERR_INVALID_ARGUMENT, "null segment input");
  const size_t need = seg_workspace_bytes(num_rows, num_slots);
  if (!ws || ws_bytes < need)
    return fail(PLORA_ERR_WORKSPACE, "segment workspace %zu < %zu bytes", ws_bytes, need);
  if (num_rows <= kSegSmallRows && num_slots <= kSegSmallSlots && num_rows * max_seq <= kSegSmallTokens) {
    PLORA_CUDA(launch_kernel(seg_small_kernel, dim3(1), dim3(1024), 0, stream, true, 0, wi, seq_lens, ranks,
                             (int32_t)num_rows, max_seq, num_slots, slot_start, token_index),
               "launch seg_small_kernel");
    return check_launch("seg_small_kernel");
  }
  SegWorkspace w = seg_workspace_carve(ws, num_rows, num_slots);
  const int64_t blocks = (num_rows + kSegRowsPerBlock - 1) / kSegRowsPerBlock;
  if (blocks > INT32_MAX) return fail(PLORA_ERR_UNSUPPORTED, "too many rows");
  // programmatic launches: each kernel waits for its predecessor before touching memory
  PLORA_CUDA(launch_kernel(seg_count_kernel, dim3((unsigned)blocks), dim3(kSegRowsPerBlock), (size_t)num_slots * 4,
                           stream, true, 0, wi, seq_lens, ranks, num_rows, max_seq, num_slots, w),
             "launch seg_count_kernel");
  int st = check_launch("seg_count_kernel");
  if (st) return st;
  if (blocks * num_slots <= kSegScanPlaceMaxInts) {  // scan and placement in one launch
    DeviceInfo* di = nullptr;
    if ((st = device_info(&di))) return st;
    const int64_t grid = std::min<int64_t>(di->sm_count, (num_rows + 31) / 32);
    PLORA_CUDA(launch_kernel(seg_scan_place_kernel, dim3((unsigned)grid), dim3(1024),
                             (size_t)(blocks * num_slots + num_slots + 1) * 4, stream, true, 0, num_rows, max_seq,
                             seq_lens, (int32_t)blocks, num_slots, w, slot_start, token_index),
               "launch seg_scan_place_kernel");
    return check_launch("seg_scan_place_kernel");
  }
  PLORA_CUDA(launch_kernel(seg_scan_kernel, dim3(1), dim3(1024), (size_t)num_slots * 4, stream, true, 0,
                           (int32_t)blocks, num_slots, w, slot_start),
             "launch seg_scan_kernel");
  if ((st = check_launch("seg_scan_kernel"))) return st;
  PLORA_CUDA(launch_kernel(seg_place_kernel, dim3((unsigned)((num_rows + 7) / 8)), dim3(256), 0, stream, true, 0,
                           num_rows, max_seq, seq_lens, (int32_t)blocks, w, slot_start, token_index),
             "launch seg_place_kernel");
  return check_launch("seg_place_kernel");
}

// Tensor-core path eligibility (16-bit types, rank tile 16/32/64, 16-byte rows).
bool tc_rank_ok(int64_t R) { return R == 16 || R == 32 || R == 64; }


// K parts of the grid-split shrink: parts of >= 2048 rows (a multiple of 32),
// at most 8 (a portable cluster).  On B200 at config-4 decode (256 tokens over
// 128 slots) that measured fastest: K = 14336 in 7 parts took 45.3 us against
// 49.7 in 8 and 65.6 in 16 (16-CTA clusters fit only ~16 at once); K = 4096 in
// 2 parts 24.8 us against 26.7 in 8.
void grid_k_parts(int64_t K, int* parts, int* part_rows) {
  int kp = (int)std::min<int64_t>(8, std::max<int64_t>(1, (K + 2047) / 2048));
  const int rows = (int)(((K + kp - 1) / kp + 31) / 32 * 32);
  *part_rows = rows;
  *parts = (int)((K + rows - 1) / rows);
}


int shrink_impl(const void* x, const void* a, void* tmp, const int32_t* ranks, SegTable seg,
                int64_t num_tokens, int64_t K, int64_t R, int32_t stack_num, int32_t dtype,
                cudaStream_t stream) {
  DeviceInfo* di = nullptr;
  int st = device_info(&di);
  if (st) return st;
  ShrinkArgs args;
  args.x = static_cast<const uint8_t*>(x);
  args.a = static_cast<const uint8_t*>(a);
  args.tmp = static_cast<uint8_t*>(tmp);
  args.ranks = ranks;
  args.seg = seg;
  args.K = (int32_t)K;
  args.R = (int32_t)R;
  args.stack_num = stack_num;
  const bool tc = dtype != PLORA_DTYPE_F32 && tc_rank_ok(R) && K % 32 == 0 &&
                  seg.num_slots <= kFastPathMaxSlots && aligned16(x) &&
                  aligned16(a) && aligned16(tmp);
  if (tc) {
    const bool bf = dtype == PLORA_DTYPE_BF16;
    if (use_weight_split(num_tokens, di)) {  // few tokens per slot: grid split
      int kp = 0, kp_rows = 0;
      grid_k_parts(K, &kp, &kp_rows);
      // rows: slots plus later 16-token tiles (few K parts, rows within a grid dimension), else slots
      const int64_t tile_rows = grid_tile_rows(num_tokens, seg.num_slots);
      const bool by_tile = kp <= kTileMaxKParts && tile_rows <= 65535;
      const dim3 grid((unsigned)kp, (unsigned)(by_tile ? tile_rows : seg.num_slots));
      // the kernel reads its inputs only after griddep_wait(): always launched programmatically
#define LAUNCH_SHRINK_GRID(RPV)                                                                    \
  PLORA_CUDA(launch_kernel(bf ? sgmv_shrink_grid_kernel<RPV, true> : sgmv_shrink_grid_kernel<RPV, false>, \
                           grid, dim3(kGridThreads), ShrinkGridCfg<RPV>::kSmemBytes, stream, true, kp, \
                           args, kp_rows, by_tile, (int)grid_later_rows(num_tokens)),              \
             "launch sgmv_shrink_grid_kernel");
      if (R == 16) {
        LAUNCH_SHRINK_GRID(16)
      } else if (R == 32) {
        LAUNCH_SHRINK_GRID(32)
      } else {
        LAUNCH_SHRINK_GRID(64)
      }
#undef LAUNCH_SHRINK_GRID
      return check_launch("sgmv_shrink_grid_kernel");
    }
    if (stream_shrink_ok(R, K, num_tokens, seg.num_slots, di)) {  // rank 16: rows through a bulk-copy ring, A in registers
      const StreamPlan plan = shrink_stream_plan(K, seg.num_slots);
      if (plan.nst >= 2) {
        // the kernel reads its inputs only after griddep_wait(): always launched programmatically
        PLORA_CUDA(launch_kernel(bf ? sgmv_shrink_stream_kernel<true, false> : sgmv_shrink_stream_kernel<false, false>,
                                 dim3(di->sm_count), dim3(kShrinkThreads), plan.smem_bytes, stream, true, 0,
                                 args, plan, ExpandArgs{}, FusedPlan{}),
                   "launch sgmv_shrink_stream_kernel");
        return check_launch("sgmv_shrink_stream_kernel");
      }
    }
    CUtensorMap map8, map1;
    const CUtensorMapSwizzle swz = R == 16   ? CU_TENSOR_MAP_SWIZZLE_32B
                                   : R == 32 ? CU_TENSOR_MAP_SWIZZLE_64B
                                             : CU_TENSOR_MAP_SWIZZLE_128B;
    if ((st = make_map_lora_a_blocks(&map8, a, dtype, (uint64_t)R, (uint64_t)K,
                                     (uint64_t)seg.num_slots, kWinBoxRows / 32, swz)) ||
        (st = make_map_lora_a_blocks(&map1, a, dtype, (uint64_t)R, (uint64_t)K,
                                     (uint64_t)seg.num_slots, 1, swz)))
      return st;
    const dim3 grid(di->sm_count), block(kMmaThreads);
    const size_t tb = tab_bytes(seg.num_slots);
    // the kernel reads its inputs only after griddep_wait(): always launched programmatically
#define LAUNCH_SHRINK(RPV)                                                                         \
  PLORA_CUDA(launch_kernel(bf ? sgmv_shrink_mma_kernel<RPV, true> : sgmv_shrink_mma_kernel<RPV, false>, \
                           grid, block, ShrinkMmaCfg<RPV>::kSmemBytes + tb, stream, true, 0, map8, map1, args), \
             "launch sgmv_shrink_mma_kernel");
    if (R == 16) {
      LAUNCH_SHRINK(16)
    } else if (R == 32) {
      LAUNCH_SHRINK(32)
    } else {
      LAUNCH_SHRINK(64)
    }
#undef LAUNCH_SHRINK
    return check_launch("sgmv_shrink_mma_kernel");
  }
  if (R > kSimtMaxRank) return fail(PLORA_ERR_UNSUPPORTED, "max_rank %lld > %d", (long long)R, kSimtMaxRank);
  const dim3 grid(di->sm_count * 8), block(kSimtThreads);
  if (dtype == PLORA_DTYPE_F32)
    sgmv_shrink_simt_kernel<float><<<grid, block, 0, stream>>>(args, seg.num_slots);
  else if (dtype == PLORA_DTYPE_BF16)
    sgmv_shrink_simt_kernel<__nv_bfloat16><<<grid, block, 0, stream>>>(args, seg.num_slots);
  else
    sgmv_shrink_simt_kernel<__half><<<grid, block, 0, stream>>>(args, seg.num_slots);
  return check_launch("sgmv_shrink_simt_kernel");
}

int expand_impl(const void* tmp, const void* b, void* y, const int32_t* ranks, const float* scales,
                SegTable seg, int64_t num_tokens, int64_t R, int64_t N, int32_t dtype,
                cudaStream_t stream, bool after_shrink = false) {
  DeviceInfo* di = nullptr;
  int st = device_info(&di);
  if (st) return st;
  ExpandArgs args;
  args.tmp = static_cast<const uint8_t*>(tmp);
  args.b = static_cast<const uint8_t*>(b);
  args.y = static_cast<uint8_t*>(y);
  args.ranks = ranks;
  args.scales = scales;
  args.seg = seg;
  args.R = (int32_t)R;
  args.N = (int32_t)N;
  const bool tc = dtype != PLORA_DTYPE_F32 && tc_rank_ok(R) && N % 64 == 0 &&
                  seg.num_slots <= kFastPathMaxSlots && aligned16(tmp) &&
                  aligned16(b) && aligned16(y);
  if (tc) {
    const bool bf = dtype == PLORA_DTYPE_BF16;
    if (use_weight_split(num_tokens, di)) {  // few tokens per slot: grid split
      // rows: slots plus later 16-token tiles (few column chunks, rows within a grid dimension), else slots
      const int64_t chunks = (N + kGridCols - 1) / kGridCols;
      const int64_t tile_rows = grid_tile_rows(num_tokens, seg.num_slots);
      const bool by_tile = chunks <= kTileMaxColChunks && tile_rows <= 65535;
      const dim3 grid((unsigned)chunks, (unsigned)(by_tile ? tile_rows : seg.num_slots));
      // programmatic only right after this library's shrink: tmp is read after griddep_wait()
#define LAUNCH_EXPAND_GRID(RPV)                                                                    \
  PLORA_CUDA(launch_kernel(bf ? sgmv_expand_grid_kernel<RPV, true> : sgmv_expand_grid_kernel<RPV, false>, \
                           grid, dim3(kGridThreads), ExpandGridCfg<RPV>::kSmemBytes, stream,       \
                           after_shrink, 0, args, by_tile, (int)grid_later_rows(num_tokens)),       \
             "launch sgmv_expand_grid_kernel");
      if (R == 16) {
        LAUNCH_EXPAND_GRID(16)
      } else if (R == 32) {
        LAUNCH_EXPAND_GRID(32)
      } else {
        LAUNCH_EXPAND_GRID(64)
      }
#undef LAUNCH_EXPAND_GRID
      return check_launch("sgmv_expand_grid_kernel");
    }
    if (stream_expand_ok(R, N, num_tokens, seg.num_slots, di)) {  // rank 16: rows through a bulk-copy ring, B in registers
      const StreamPlan plan = expand_stream_plan(N, seg.num_slots);
      if (plan.smem_bytes <= (uint32_t)kStreamSmemLimit) {
        // programmatic only right after this library's shrink (after_shrink): the kernel
        // reads the segment table and LoRA-B before griddep_wait(), tmp after it; y is
        // only added to, after tmp
        PLORA_CUDA(launch_kernel(bf ? sgmv_expand_stream_kernel<true> : sgmv_expand_stream_kernel<false>,
                                 dim3(di->sm_count), dim3(kStreamThreads), plan.smem_bytes, stream,
                                 after_shrink, 0, args, plan),
                   "launch sgmv_expand_stream_kernel");
        return check_launch("sgmv_expand_stream_kernel");
      }
    }
    CUtensorMap mapn, map1;
    const uint32_t box = R == 16 ? ExpandMmaCfg<16>::kBoxChunks
                         : R == 32 ? ExpandMmaCfg<32>::kBoxChunks
                                   : ExpandMmaCfg<64>::kBoxChunks;
    if ((st = make_map_lora_b_chunks(&mapn, b, dtype, (uint64_t)R, (uint64_t)N,
                                     (uint64_t)seg.num_slots, box)) ||
        (st = make_map_lora_b_chunks(&map1, b, dtype, (uint64_t)R, (uint64_t)N,
                                     (uint64_t)seg.num_slots, 1)))
      return st;
    const dim3 grid(di->sm_count), block(kMmaThreads);
    const size_t tb = tab_bytes(seg.num_slots);
    // programmatic only right after this library's shrink (after_shrink): the kernel reads
    // the segment table, LoRA-B and y before griddep_wait(), tmp after it
#define LAUNCH_EXPAND(RPV)                                                                         \
  PLORA_CUDA(launch_kernel(bf ? sgmv_expand_mma_kernel<RPV, true> : sgmv_expand_mma_kernel<RPV, false>, \
                           grid, block, ExpandMmaCfg<RPV>::kSmemBytes + tb, stream, after_shrink, 0, mapn, \
                           map1, args),                                                            \
             "launch sgmv_expand_mma_kernel");
    if (R == 16) {
      LAUNCH_EXPAND(16)
    } else if (R == 32) {
      LAUNCH_EXPAND(32)
    } else {
      LAUNCH_EXPAND(64)
    }
#undef LAUNCH_EXPAND
    return check_launch("sgmv_expand_mma_kernel");
  }
  if (R > kSimtMaxRank) return fail(PLORA_ERR_UNSUPPORTED, "max_rank %lld > %d", (long long)R, kSimtMaxRank);
  const dim3 grid(di->sm_count * 8), block(kSimtThreads);
  if (dtype == PLORA_DTYPE_F32)
    sgmv_expand_simt_kernel<float><<<grid, block, 0, stream>>>(args, seg.num_slots);
  else if (dtype == PLORA_DTYPE_BF16)
    sgmv_expand_simt_kernel<__nv_bfloat16><<<grid, block, 0, stream>>>(args, seg.num_slots);
  else
    sgmv_expand_simt_kernel<__half><<<grid, block, 0, stream>>>(args, seg.num_slots);
  return check_launch("sgmv_expand_simt_kernel");
}

int check_common(int32_t dtype, int32_t num_slots, int64_t max_rank) {
  if (!valid_dtype(dtype)) return fail(PLORA_ERR_INVALID_ARGUMENT, "unknown dtype %d", dtype);
  if (num_slots < 1 || num_slots > kSegMaxSlots)
    return fail(PLORA_ERR_UNSUPPORTED, "num_slots %d outside [1, %d]", num_slots, kSegMaxSlots);
  if (max_rank < 1) return fail(PLORA_ERR_INVALID_ARGUMENT, "max_rank must be >= 1");
  return PLORA_OK;
}

FwdWorkspace carve_fwd(void* ws, int64_t num_rows, int64_t max_seq, int32_t num_slots) {
  FwdWorkspace f;
  char* p = static_cast<char*>(ws);
  f.seg = seg_workspace_carve(p, num_rows, num_slots);
  p += seg_workspace_bytes(num_rows, num_slots);
  f.slot_start = reinterpret_cast<int32_t*>(p);
  p += align256((size_t)(num_slots + 1) * 4);
  f.token_index = reinterpret_cast<int32_t*>(p);
  return f;
}

// Device address of `bytes` (> 0) bytes of host memory that a kernel may read
// and write over PCIe: page-locked and mapped at both ends, as one range.
int mapped_host_range(const void* p, int64_t bytes, const char* what, const uint8_t** dev) {
  cudaPointerAttributes a = {}, b = {};
  const void* last = static_cast<const uint8_t*>(p) + (bytes - 1);
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess || cudaPointerGetAttributes(&b, last) != cudaSuccess) {
    cudaGetLastError();
    return fail(PLORA_ERR_INVALID_ARGUMENT, "%s: pointer attributes unavailable", what);
  }
  if (a.type != cudaMemoryTypeHost || b.type != cudaMemoryTypeHost || !a.devicePointer || !b.devicePointer)
    return fail(PLORA_ERR_INVALID_ARGUMENT, "%s must be page-locked, mapped host memory", what);
  const uint8_t* d0 = static_cast<const uint8_t*>(a.devicePointer);
  if (static_cast<const uint8_t*>(b.devicePointer) - d0 != bytes - 1)
    return fail(PLORA_ERR_INVALID_ARGUMENT, "%s is not one mapped range", what);
  *dev = d0;
  return PLORA_OK;
}

int device_range(const void* p, int64_t bytes, const char* what) {
  cudaPointerAttributes a = {}, b = {};
  const void* last = static_cast<const uint8_t*>(p) + (bytes - 1);
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess || cudaPointerGetAttributes(&b, last) != cudaSuccess) {
    cudaGetLastError();
    return fail(PLORA_ERR_INVALID_ARGUMENT, "%s: pointer attributes unavailable", what);
  }
  const bool ok = (a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged) && a.type == b.type;
  if (!ok) return fail(PLORA_ERR_INVALID_ARGUMENT, "%s must be device memory", what);
  return PLORA_OK;
}

// Both directions of the token-row copy: arguments checked on the host, then
// one programmatic launch of token_rows_copy_kernel.
int token_rows_impl(const void* host_rows, void* device_rows, bool to_host, int64_t row_bytes, int64_t num_tokens,
                    const int32_t* slot_start, const int32_t* token_index, int32_t num_slots, void* stream) {
  g_last_error.clear();
  if (row_bytes < 16 || row_bytes % 16 || num_tokens < 0)
    return fail(PLORA_ERR_INVALID_ARGUMENT, "row_bytes must be a positive multiple of 16, num_tokens >= 0");
  if (num_slots < 1 || num_slots > kSegMaxSlots)
    return fail(PLORA_ERR_UNSUPPORTED, "num_slots %d outside [1, %d]", num_slots, kSegMaxSlots);
  if (num_tokens > (int64_t)INT32_MAX) return fail(PLORA_ERR_UNSUPPORTED, "num_tokens exceeds int32 token ids");
  if (row_bytes > INT64_MAX / std::max<int64_t>(num_tokens, 1))
    return fail(PLORA_ERR_INVALID_ARGUMENT, "num_tokens * row_bytes overflows");
  if (num_tokens == 0) return PLORA_OK;
  if (!host_rows || !device_rows || !slot_start || !token_index)
    return fail(PLORA_ERR_INVALID_ARGUMENT, "null pointer");
  if (reinterpret_cast<uintptr_t>(host_rows) % 16 || reinterpret_cast<uintptr_t>(device_rows) % 16)
    return fail(PLORA_ERR_INVALID_ARGUMENT, "row buffers must be 16-byte aligned");
  const int64_t bytes = num_tokens * row_bytes;
  const uint8_t* host_dev = nullptr;
  int st = mapped_host_range(host_rows, bytes, "host_rows", &host_dev);
  if (st) return st;
  st = device_range(device_rows, bytes, "device_rows");
  if (st) return st;
  DeviceInfo* di = nullptr;
  st = device_info(&di);
  if (st) return st;
  const uint8_t* dev_rows = static_cast<const uint8_t*>(device_rows);
  const uint8_t* src = to_host ? dev_rows : host_dev;
  uint8_t* dst = const_cast<uint8_t*>(to_host ? host_dev : dev_rows);
  // a plain launch: the rows' producers typically finish on another stream (events)
  PLORA_CUDA(launch_kernel(token_rows_copy_kernel, dim3((unsigned)(2 * di->sm_count)), dim3(kRowsThreads), 0,
                           static_cast<cudaStream_t>(stream), false, 0, src, dst, row_bytes, num_tokens, slot_start,
                           token_index, num_slots),
             "launch token_rows_copy_kernel");
  return PLORA_OK;
}

}  // namespace

extern "C" {

const char* plora_version(void) { return "polylora_b200 0.1.0 (sm_100a)"; }

const char* plora_status_string(int status) {
  switch (status) {
    case PLORA_OK: return "ok";
    case PLORA_ERR_INVALID_ARGUMENT: return "invalid argument";
    case PLORA_ERR_UNSUPPORTED: return "unsupported";
    case PLORA_ERR_CUDA: return "CUDA error";
    case PLORA_ERR_WORKSPACE: return "workspace too small";
    case PLORA_ERR_DEVICE: return "device status raised";
    default: return "unknown status";
  }
}

const char* plora_last_error(void) { return g_last_error.c_str(); }

int64_t plora_weight_split_tokens_per_sm(int64_t value) {
  return value >= 0 ? g_wsplit_tokens_per_sm.exchange(value) : g_wsplit_tokens_per_sm.load();
}

int32_t plora_stream_kernels(int32_t value) {
  return value >= 0 ? g_stream_kernels.exchange(value > 2 ? 2 : value) : g_stream_kernels.load();
}

int plora_set_wait_limit_ns(uint64_t limit_ns, uint64_t* previous) {
  g_last_error.clear();
  uint64_t old = 0;
  PLORA_CUDA(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
  PLORA_CUDA(cudaMemcpyFromSymbol(&old, g_wait_limit_ns, sizeof(old)), "read wait limit");
  PLORA_CUDA(cudaMemcpyToSymbol(g_wait_limit_ns, &limit_ns, sizeof(limit_ns)), "set wait limit");
  if (previous) *previous = old;
  return PLORA_OK;
}

int plora_device_status(int32_t* status_out, int32_t clear) {
  int v = 0;
  PLORA_CUDA(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
  PLORA_CUDA(cudaMemcpyFromSymbol(&v, g_device_status, sizeof(int)), "read device status");
  if (clear) {
    const int zero = 0;
    PLORA_CUDA(cudaMemcpyToSymbol(g_device_status, &zero, sizeof(int)), "clear device status");
  }
  if (status_out) *status_out = v;
  return v ? fail(PLORA_ERR_DEVICE, "device status 0x%x", v) : PLORA_OK;
}

size_t plora_workspace_size(int64_t num_rows, int64_t max_seq, int32_t num_slots) {
  if (!token_count_ok(num_rows, max_seq) || num_slots < 1 || num_slots > kSegMaxSlots) return 0;
  return fwd_workspace_bytes(num_rows, max_seq, num_slots);
}

int plora_build_segments(const int64_t* weight_indices, const int32_t* seq_lens,
                         const int32_t* lora_ranks, int64_t num_rows, int64_t max_seq,
                         int32_t num_slots, int32_t* slot_start, int32_t* token_index,
                         void* workspace, size_t workspace_size, void* stream) {
  g_last_error.clear();
  return build_segments(weight_indices, seq_lens, lora_ranks, num_rows, max_seq, num_slots,
                        slot_start, token_index, workspace, workspace_size,
                        static_cast<cudaStream_t>(stream));
}

int plora_gather_token_rows(const void* host_rows, void* device_rows, int64_t row_bytes, int64_t num_tokens,
                            const int32_t* slot_start, const int32_t* token_index, int32_t num_slots,
                            void* stream) {
  return token_rows_impl(host_rows, device_rows, false, row_bytes, num_tokens, slot_start, token_index, num_slots,
                         stream);
}

int plora_scatter_token_rows(const void* device_rows, void* host_rows, int64_t row_bytes, int64_t num_tokens,
                             const int32_t* slot_start, const int32_t* token_index, int32_t num_slots,
                             void* stream) {
  return token_rows_impl(host_rows, const_cast<void*>(device_rows), true, row_bytes, num_tokens, slot_start,
                         token_index, num_slots, stream);
}

int plora_check_right_padded(const void* mask, int32_t mask_elem_bytes, int32_t mask_is_float,
                             const int64_t* seq_lens, int64_t rows, int64_t width, void* stream) {
  g_last_error.clear();
  const bool size_ok = mask_elem_bytes == 1 || mask_elem_bytes == 2 || mask_elem_bytes == 4 || mask_elem_bytes == 8;
  if (rows < 0 || width < 0 || !size_ok || (mask_is_float && mask_elem_bytes == 1))
    return fail(PLORA_ERR_INVALID_ARGUMENT, "mask shape or element type");
  if (rows > INT32_MAX) return fail(PLORA_ERR_UNSUPPORTED, "more than 2^31-1 mask rows");
  if (rows == 0 || width == 0) return PLORA_OK;
  if (!mask || !seq_lens) return fail(PLORA_ERR_INVALID_ARGUMENT, "null pointer");
  if (reinterpret_cast<uintptr_t>(mask) % mask_elem_bytes)
    return fail(PLORA_ERR_INVALID_ARGUMENT, "mask not aligned to its element size");
  mask_padding_kernel<<<(unsigned)rows, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(mask), mask_elem_bytes, mask_is_float ? 1 : 0, seq_lens, width);
  return check_launch("mask_padding_kernel");
}

int plora_flat_schedule(const int32_t* seq_lens, const int32_t* n_eff, int64_t num_rows,
                        int32_t block_m, int32_t block_n, int32_t* cum_tiles,
                        int32_t* num_n_tiles, void* stream) {
  g_last_error.clear();
  if (num_rows < 0 || block_m < 1 || block_n < 1 || !cum_tiles)
    return fail(PLORA_ERR_INVALID_ARGUMENT, "flat schedule arguments");
  if (num_rows > 0 && (!seq_lens || !n_eff || !num_n_tiles))
    return fail(PLORA_ERR_INVALID_ARGUMENT, "null flat schedule input");
  flat_schedule_kernel<<<1, 1024, 0, static_cast<cudaStream_t>(stream)>>>(
      seq_lens, n_eff, num_rows, block_m, block_n, cum_tiles, num_n_tiles);
  return check_launch("flat_schedule_kernel");
}

int plora_sgmv_shrink(const void* x, const void* lora_a, void* tmp, const int32_t* lora_ranks,
                      const int32_t* slot_start, const int32_t* token_index, int64_t num_tokens,
                      int64_t in_features, int64_t max_rank, int32_t num_slots, int32_t stack_num,
                      int32_t dtype, void* stream) {
  g_last_error.clear();
  int st = check_common(dtype, num_slots, max_rank);
  if (st) return st;
  if (in_features < 1 || in_features > INT32_MAX || stack_num < 1)
    return fail(PLORA_ERR_INVALID_ARGUMENT, "in_features/stack_num");
  if (num_tokens == 0) return PLORA_OK;
  if (!x || !lora_a || !tmp || !lora_ranks || !slot_start || !token_index)
    return fail(PLORA_ERR_INVALID_ARGUMENT, "null pointer");
  SegTable seg{slot_start, token_index, num_slots};
  if (num_tokens > (int64_t)INT32_MAX)
    return fail(PLORA_ERR_UNSUPPORTED, "num_tokens exceeds int32 token ids");
  return shrink_impl(x, lora_a, tmp, lora_ranks, seg, num_tokens, in_features, max_rank, stack_num,
                     dtype, static_cast<cudaStream_t>(stream));
}

int plora_sgmv_expand(const void* tmp, const void* lora_b, void* y, const int32_t* lora_ranks,
                      const float* scalings, const int32_t* slot_start, const int32_t* token_index,
                      int64_t num_tokens, int64_t max_rank, int64_t out_features,
                      int32_t num_slots, int32_t dtype, void* stream) {
  g_last_error.clear();
  int st = check_common(dtype, num_slots, max_rank);
  if (st) return st;
  if (out_features < 1 || out_features > INT32_MAX)
    return fail(PLORA_ERR_INVALID_ARGUMENT, "out_features");
  if (num_tokens == 0) return PLORA_OK;
  if (!tmp || !lora_b || !y || !lora_ranks || !scalings || !slot_start || !token_index)
    return fail(PLORA_ERR_INVALID_ARGUMENT, "null pointer");
  SegTable seg{slot_start, token_index, num_slots};
  return expand_impl(tmp, lora_b, y, lora_ranks, scalings, seg, num_tokens, max_rank, out_features,
                     dtype, static_cast<cudaStream_t>(stream));
}

// The fused stream kernel for plora_sgmv_shrink_expand: rank 16, 16-bit types,
// K and N multiples of 512 up to 4096, many tokens, and an expand phase that
// fits the shrink's shared memory.  *launched = false leaves the call to the
// two kernels.
int fused_impl(const void* x, const void* a, void* tmp, const void* b, void* y, const int32_t* ranks,
               const float* scales, SegTable seg, int64_t num_tokens, int64_t K, int64_t R, int64_t N, int32_t dtype,
               cudaStream_t stream, bool* launched) {
  *launched = false;
  if (g_stream_kernels.load(std::memory_order_relaxed) != 2 || dtype == PLORA_DTYPE_F32 || R != kStreamRank ||
      seg.num_slots > kFastPathMaxSlots || !aligned16(x) || !aligned16(a) || !aligned16(tmp) || !aligned16(b) ||
      !aligned16(y) || N % 512 != 0 || N > kStreamMaxDim)
    return PLORA_OK;
  DeviceInfo* di = nullptr;
  int st = device_info(&di);
  if (st) return st;
  if (use_weight_split(num_tokens, di) || !stream_shrink_ok(R, K, num_tokens, seg.num_slots, di)) return PLORA_OK;
  StreamPlan plan;
  FusedPlan fp;
  if (!fused_stream_plan(K, N, seg.num_slots, plan, fp)) return PLORA_OK;
  ShrinkArgs sa;
  sa.x = static_cast<const uint8_t*>(x);
  sa.a = static_cast<const uint8_t*>(a);
  sa.tmp = static_cast<uint8_t*>(tmp);
  sa.ranks = ranks;
  sa.seg = seg;
  sa.K = (int32_t)K;
  sa.R = (int32_t)R;
  sa.stack_num = 1;
  ExpandArgs ea;
  ea.tmp = static_cast<const uint8_t*>(tmp);
  ea.b = static_cast<const uint8_t*>(b);
  ea.y = static_cast<uint8_t*>(y);
  ea.ranks = ranks;
  ea.scales = scales;
  ea.seg = seg;
  ea.R = (int32_t)R;
  ea.N = (int32_t)N;
  const bool bf = dtype == PLORA_DTYPE_BF16;
  // programmatic like the shrink: it reads its inputs only after griddep_wait()
  PLORA_CUDA(launch_kernel(bf ? sgmv_shrink_stream_kernel<true, true> : sgmv_shrink_stream_kernel<false, true>,
                           dim3(di->sm_count), dim3(kShrinkThreads), plan.smem_bytes, stream, true, 0, sa, plan,
                           ea, fp),
             "launch fused sgmv_shrink_stream_kernel");
  *launched = true;
  return check_launch("fused sgmv_shrink_stream_kernel");
}

int plora_sgmv_shrink_expand(const void* x, const void* lora_a, void* tmp, const void* lora_b,
                             void* y, const int32_t* lora_ranks, const float* scalings,
                             const int32_t* slot_start, const int32_t* token_index,
                             int64_t num_tokens, int64_t in_features, int64_t max_rank,
                             int64_t out_features, int32_t num_slots, int32_t dtype,
                             void* stream) {
  g_last_error.clear();
  int st = check_common(dtype, num_slots, max_rank);
  if (st) return st;
  if (in_features < 1 || in_features > INT32_MAX || out_features < 1 || out_features > INT32_MAX)
    return fail(PLORA_ERR_INVALID_ARGUMENT, "in_features/out_features");
  if (num_tokens == 0) return PLORA_OK;
  if (!x || !lora_a || !tmp || !lora_b || !y || !lora_ranks || !scalings || !slot_start ||
      !token_index)
    return fail(PLORA_ERR_INVALID_ARGUMENT, "null pointer");
  if (num_tokens > (int64_t)INT32_MAX)
    return fail(PLORA_ERR_UNSUPPORTED, "num_tokens exceeds int32 token ids");
  SegTable seg{slot_start, token_index, num_slots};
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  bool fused = false;
  if ((st = fused_impl(x, lora_a, tmp, lora_b, y, lora_ranks, scalings, seg, num_tokens, in_features, max_rank,
                       out_features, dtype, s, &fused)) || fused)
    return st;
  if ((st = shrink_impl(x, lora_a, tmp, lora_ranks, seg, num_tokens, in_features, max_rank, 1,
                        dtype, s)))
    return st;
  return expand_impl(tmp, lora_b, y, lora_ranks, scalings, seg, num_tokens, max_rank, out_features,
                     dtype, s, /*after_shrink=*/true);
}

int plora_sgmv_a_fwd(const void* x, const void* lora_a, void* tmp, const int32_t* seq_lens,
                     const int64_t* weight_indices, const int32_t* lora_ranks, int64_t num_rows,
                     int64_t max_seq, int64_t in_features, int64_t max_rank, int32_t num_slots,
                     int32_t stack_num, int32_t dtype, void* workspace, size_t workspace_size,
                     void* stream) {
  g_last_error.clear();
  int st = check_common(dtype, num_slots, max_rank);
  if (st) return st;
  if (!token_count_ok(num_rows, max_seq))
    return fail(PLORA_ERR_UNSUPPORTED, "num_rows %lld x max_seq %lld: negative or beyond int32 token ids",
                (long long)num_rows, (long long)max_seq);
  if (num_rows == 0 || max_seq == 0) return PLORA_OK;  // sgmv.py:159-160
  const size_t need = fwd_workspace_bytes(num_rows, max_seq, num_slots);
  if (!workspace || workspace_size < need)
    return fail(PLORA_ERR_WORKSPACE, "workspace %zu < %zu bytes", workspace_size, need);
  FwdWorkspace w = carve_fwd(workspace, num_rows, max_seq, num_slots);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if ((st = build_segments(weight_indices, seq_lens, lora_ranks, num_rows, max_seq, num_slots,
                           w.slot_start, w.token_index, workspace, workspace_size, s)))
    return st;
  return plora_sgmv_shrink(x, lora_a, tmp, lora_ranks, w.slot_start, w.token_index,
                           num_rows * max_seq, in_features, max_rank, num_slots, stack_num, dtype,
                           stream);
}

int plora_sgmv_b_fwd(const void* tmp, const void* lora_b, void* y, const int32_t* seq_lens,
                     const int64_t* weight_indices, const int32_t* lora_ranks,
                     const float* scalings, int64_t num_rows, int64_t max_seq, int64_t max_rank,
                     int64_t out_features, int32_t num_slots, int32_t dtype, void* workspace,
                     size_t workspace_size, void* stream) {
  g_last_error.clear();
  int st = check_common(dtype, num_slots, max_rank);
  if (st) return st;
  if (!token_count_ok(num_rows, max_seq))
    return fail(PLORA_ERR_UNSUPPORTED, "num_rows %lld x max_seq %lld: negative or beyond int32 token ids",
                (long long)num_rows, (long long)max_seq);
  if (num_rows == 0 || max_seq == 0) return PLORA_OK;  // sgmv.py:314-315
  const size_t need = fwd_workspace_bytes(num_rows, max_seq, num_slots);
  if (!workspace || workspace_size < need)
    return fail(PLORA_ERR_WORKSPACE, "workspace %zu < %zu bytes", workspace_size, need);
  FwdWorkspace w = carve_fwd(workspace, num_rows, max_seq, num_slots);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if ((st = build_segments(weight_indices, seq_lens, lora_ranks, num_rows, max_seq, num_slots,
                           w.slot_start, w.token_index, workspace, workspace_size, s)))
    return st;
  return plora_sgmv_expand(tmp, lora_b, y, lora_ranks, scalings, w.slot_start, w.token_index,
                           num_rows * max_seq, max_rank, out_features, num_slots, dtype, stream);
}

int plora_slot_fill(const plora_slot_module* modules, int32_t num_modules, int32_t slot,
                    int32_t num_slots, int64_t max_rank, int32_t dtype, const void* host_image,
                    size_t image_bytes, void* staging, size_t staging_bytes, void* stream) {
  g_last_error.clear();
  if (!valid_dtype(dtype)) return fail(PLORA_ERR_INVALID_ARGUMENT, "unknown dtype %d", dtype);
  if (num_modules < 0 || slot < 0 || slot >= num_slots || max_rank < 1)
    return fail(PLORA_ERR_INVALID_ARGUMENT, "slot %d of %d, %d modules", slot, num_slots,
                num_modules);
  if (num_modules == 0) return PLORA_OK;
  if (!modules || !host_image || !staging)
    return fail(PLORA_ERR_INVALID_ARGUMENT, "null pointer");
  if (image_bytes < (size_t)num_modules * sizeof(plora_slot_record))
    return fail(PLORA_ERR_INVALID_ARGUMENT, "image smaller than its records");
  if (staging_bytes < image_bytes)
    return fail(PLORA_ERR_WORKSPACE, "staging %zu < image %zu bytes", staging_bytes, image_bytes);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  PLORA_CUDA(cudaMemcpyAsync(staging, host_image, image_bytes, cudaMemcpyHostToDevice, s),
             "slot image copy");
  const dim3 grid(64, (unsigned)num_modules), block(256);
  const uint8_t* img = static_cast<const uint8_t*>(staging);
  const int64_t nbytes = (int64_t)image_bytes;
  if (elem_size(dtype) == 4)
    slot_fill_kernel<float><<<grid, block, 0, s>>>(modules, num_modules, slot, max_rank, img, nbytes);
  else if (dtype == PLORA_DTYPE_BF16)
    slot_fill_kernel<__nv_bfloat16><<<grid, block, 0, s>>>(modules, num_modules, slot, max_rank, img, nbytes);
  else
    slot_fill_kernel<__half><<<grid, block, 0, s>>>(modules, num_modules, slot, max_rank, img, nbytes);
  return check_launch("slot_fill_kernel");
}

// Device address of g_noalloc_scratch, looked up once per device and CUDA
// context with that device current (the first plora_sgmv_a_fwd_noalloc call
// there).  The cache is keyed on the context's unique id: after
// cudaDeviceReset the module is loaded again in a new context, and the array
// may live at another address.
namespace {
struct NoallocScratch {
  unsigned long long ctx_id = 0;
  void* ptr = nullptr;
};
NoallocScratch g_noalloc[kMaxDevices];
std::mutex g_noalloc_mu;

// Unique id of the calling thread's current CUDA context (0 if unavailable).
unsigned long long current_context_id() {
  using GetCurrent = CUresult (*)(CUcontext*);
  using GetId = CUresult (*)(CUcontext, unsigned long long*);
  static GetCurrent get_current = nullptr;
  static GetId get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<GetCurrent>(p);
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<GetId>(p);
  });
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (!get_current || !get_id || get_current(&ctx) != CUDA_SUCCESS || !ctx || get_id(ctx, &id) != CUDA_SUCCESS)
    return 0;
  return id;
}

int noalloc_scratch(void** out) {
  int dev = 0;
  PLORA_CUDA(cudaGetDevice(&dev), "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(PLORA_ERR_UNSUPPORTED, "device ordinal %d", dev);
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  NoallocScratch& e = g_noalloc[dev];
  const unsigned long long id = current_context_id();  // 0 before the runtime set one up
  if (!e.ptr || id == 0 || e.ctx_id != id) {
    void* p = nullptr;
    // also makes the runtime's context for `dev` current on this thread
    PLORA_CUDA(cudaGetSymbolAddress(&p, g_noalloc_scratch), "cudaGetSymbolAddress(noalloc scratch)");
    e.ptr = p;
    e.ctx_id = current_context_id();
  }
  *out = e.ptr;
  return PLORA_OK;
}
}  // namespace

extern "C" int plora_sgmv_a_fwd_noalloc(const void* x, const void* lora_a, void* tmp,
                                        const int32_t* seq_lens, const int64_t* weight_indices,
                                        const int32_t* lora_ranks, int64_t num_rows,
                                        int64_t max_seq, int64_t in_features, int64_t max_rank,
                                        int32_t num_slots, int32_t stack_num, int32_t dtype,
                                        void* stream) {
  g_last_error.clear();
  int st = check_common(dtype, num_slots, max_rank);
  if (st) return st;
  if (num_rows < 0 || max_seq < 0) return fail(PLORA_ERR_INVALID_ARGUMENT, "negative num_rows/max_seq");
  if (!token_count_ok(num_rows, max_seq))
    return fail(PLORA_ERR_UNSUPPORTED, "num_rows %lld x max_seq %lld exceeds int32 token ids",
                (long long)num_rows, (long long)max_seq);
  if (num_rows == 0 || max_seq == 0) return PLORA_OK;
  const size_t need = fwd_workspace_bytes(num_rows, max_seq, num_slots);
  if (need > (size_t)PLORA_NOALLOC_SCRATCH_BYTES)
    return fail(PLORA_ERR_UNSUPPORTED,
                "batch needs %zu bytes of scratch; the static scratch of plora_sgmv_a_fwd_noalloc "
                "holds %u bytes (use plora_sgmv_a_fwd with a workspace)",
                need, (unsigned)PLORA_NOALLOC_SCRATCH_BYTES);
  void* scratch = nullptr;
  if ((st = noalloc_scratch(&scratch))) return st;
  FwdWorkspace w = carve_fwd(scratch, num_rows, max_seq, num_slots);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if ((st = build_segments(weight_indices, seq_lens, lora_ranks, num_rows, max_seq, num_slots,
                           w.slot_start, w.token_index, scratch, need, s)))
    return st;
  return plora_sgmv_shrink(x, lora_a, tmp, lora_ranks, w.slot_start, w.token_index,
                           num_rows * max_seq, in_features, max_rank, num_slots, stack_num, dtype,
                           stream);
}

}  // extern "C"
