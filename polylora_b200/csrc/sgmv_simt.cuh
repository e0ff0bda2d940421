// SGMV shrink / expand on the CUDA cores, fp32 accumulation.  Used for fp32
// activations (fp32 FFMA keeps the 1e-5 bound that TF32 tensor cores would
// not) and for bf16/fp16 shapes outside the tensor-core path (max_rank not in
// {16, 32, 64}, feature sizes not a multiple of 8, unaligned pointers).
// Same segment table and semantics as the tensor-core kernels.
#pragma once

#include "common.cuh"
#include "sgmv_common.cuh"

namespace plora {

template <typename T>
struct Cvt;
template <>
struct Cvt<float> {
  __device__ static __forceinline__ float f(float v) { return v; }
  __device__ static __forceinline__ float t(float v) { return v; }
};
template <>
struct Cvt<__half> {
  __device__ static __forceinline__ float f(__half v) { return __half2float(v); }
  __device__ static __forceinline__ __half t(float v) { return __float2half_rn(v); }
};
template <>
struct Cvt<__nv_bfloat16> {
  __device__ static __forceinline__ float f(__nv_bfloat16 v) { return __bfloat162float(v); }
  __device__ static __forceinline__ __nv_bfloat16 t(float v) { return __float2bfloat16_rn(v); }
};

constexpr int kSimtThreads = 256;
constexpr int kSimtMaxRank = 256;

// One block per active token (grid-stride over the segment table); each
// thread accumulates 32 output columns at a time over a strided slice of K,
// then a block reduction produces the column sums.
template <typename T>
__global__ void __launch_bounds__(kSimtThreads) sgmv_shrink_simt_kernel(const ShrinkArgs args,
                                                                        int32_t num_slots_a) {
  __shared__ float red[kSimtThreads / 32][32];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int64_t total = __ldg(args.seg.slot_start + args.seg.num_slots);
  const T* x = reinterpret_cast<const T*>(args.x);
  const T* a = reinterpret_cast<const T*>(args.a);
  T* tmp = reinterpret_cast<T*>(args.tmp);
  const int K = args.K, R = args.R;
  for (int64_t pos = blockIdx.x; pos < total; pos += gridDim.x) {
    const int s = slot_of_position(args.seg.slot_start, args.seg.num_slots, pos);
    const int rank = __ldg(args.ranks + s);
    if (rank <= 0 || s >= num_slots_a) continue;
    const int n_eff = min(rank * args.stack_num, R);
    const int64_t tok = __ldg(args.seg.token_index + pos);
    const T* xr = x + tok * K;
    const T* as = a + (int64_t)s * K * R;
    T* out = tmp + tok * R;
    for (int jb = 0; jb < R; jb += 32) {
      float acc[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) acc[j] = 0.f;
      if (jb < n_eff) {
        for (int k = threadIdx.x; k < K; k += kSimtThreads) {
          const float xv = Cvt<T>::f(xr[k]);
          const T* ar = as + (int64_t)k * R + jb;
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (jb + j < n_eff) acc[j] = fmaf(xv, Cvt<T>::f(ar[j]), acc[j]);
        }
      }
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        float v = acc[j];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lane == 0) red[warp][j] = v;
      }
      __syncthreads();
      if (threadIdx.x < 32) {
        const int j = jb + threadIdx.x;
        float v = 0.f;
#pragma unroll
        for (int w = 0; w < kSimtThreads / 32; ++w) v += red[w][threadIdx.x];
        if (j < R) out[j] = Cvt<T>::t(j < n_eff ? v : 0.f);
      }
      __syncthreads();
    }
  }
}

// One block per active token: tmp row staged in shared memory, each thread
// produces output columns n = tid + k*blockDim and adds them into y.
template <typename T>
__global__ void __launch_bounds__(kSimtThreads) sgmv_expand_simt_kernel(const ExpandArgs args,
                                                                        int32_t num_slots_b) {
  __shared__ float trow[kSimtMaxRank];
  const int64_t total = __ldg(args.seg.slot_start + args.seg.num_slots);
  const T* tmp = reinterpret_cast<const T*>(args.tmp);
  const T* b = reinterpret_cast<const T*>(args.b);
  T* y = reinterpret_cast<T*>(args.y);
  const int R = args.R, N = args.N;
  for (int64_t pos = blockIdx.x; pos < total; pos += gridDim.x) {
    const int s = slot_of_position(args.seg.slot_start, args.seg.num_slots, pos);
    const int rank = __ldg(args.ranks + s);
    if (rank <= 0 || s >= num_slots_b) continue;
    const int kr = min(rank, R);
    const float scale = __ldg(args.scales + s);
    const int64_t tok = __ldg(args.seg.token_index + pos);
    __syncthreads();
    for (int k = threadIdx.x; k < kr; k += kSimtThreads) trow[k] = Cvt<T>::f(tmp[tok * R + k]);
    __syncthreads();
    const T* bs = b + (int64_t)s * R * N;
    T* yr = y + tok * N;
    for (int n = threadIdx.x; n < N; n += kSimtThreads) {
      float acc = 0.f;
      for (int k = 0; k < kr; ++k) acc = fmaf(trow[k], Cvt<T>::f(bs[(int64_t)k * N + n]), acc);
      yr[n] = Cvt<T>::t(Cvt<T>::f(yr[n]) + scale * acc);
    }
  }
}

// Slot refill: every module's slot region rewritten from the staged adapter
// image (zero padding past the adapter's rank, rank/scale scalars).  The image
// holds each module's factors as PEFT stores them (A rank x in, B out x rank),
// so the host does no transposes; this kernel writes them transposed into the
// slot layouts (K x R, R x N).  Mirrors src/polylora/cache.py:108-115 (zero on
// evict) and 119-150 (load, which transposes on the host).  A record whose A or
// B block does not lie inside the image's `image_bytes` (or is not aligned to
// the element size) is not read: the module is filled as rank 0 and
// PLORA_DEV_IMAGE_RANGE is raised.
template <typename T>
__global__ void __launch_bounds__(256) slot_fill_kernel(const plora_slot_module* __restrict__ mods,
                                                         int32_t num_modules, int32_t slot,
                                                         int64_t R, const uint8_t* __restrict__ image,
                                                         int64_t image_bytes) {
  const int m = blockIdx.y;
  if (m >= num_modules) return;
  const plora_slot_module mod = mods[m];
  const plora_slot_record rec = reinterpret_cast<const plora_slot_record*>(image)[m];
  int64_t r = rec.rank;
  r = r < 0 ? 0 : (r > R ? R : r);
  const int64_t K = mod.in_features, N = mod.out_features;
  if (r > 0) {
    const int64_t esz = (int64_t)sizeof(T);
    const bool inside = rec.a_offset >= 0 && rec.b_offset >= 0 && rec.a_offset % esz == 0 &&
                        rec.b_offset % esz == 0 && rec.a_offset <= image_bytes &&
                        rec.b_offset <= image_bytes && r * K * esz <= image_bytes - rec.a_offset &&
                        r * N * esz <= image_bytes - rec.b_offset;
    if (!inside) {
      if (blockIdx.x == 0 && threadIdx.x == 0) raise_status(PLORA_DEV_IMAGE_RANGE);
      r = 0;
    }
  }
  const int64_t nA = K * R, nB = R * N;
  T* A = reinterpret_cast<T*>(mod.lora_a) + (int64_t)slot * nA;
  T* B = reinterpret_cast<T*>(mod.lora_b) + (int64_t)slot * nB;
  const T* srcA = reinterpret_cast<const T*>(image + rec.a_offset);
  const T* srcB = reinterpret_cast<const T*>(image + rec.b_offset);
  const T zero = Cvt<T>::t(0.f);
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nA + nB; i += stride) {
    if (i < nA) {
      const int64_t k = i / R, j = i - k * R;
      A[i] = (j < r) ? srcA[j * K + k] : zero;
    } else {
      const int64_t i2 = i - nA;
      const int64_t j = i2 / N, n = i2 - j * N;
      B[i2] = (j < r) ? srcB[n * r + j] : zero;
    }
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    mod.ranks[slot] = (int32_t)r;
    mod.scales[slot] = r > 0 ? rec.scale : 0.f;
  }
}

}  // namespace plora
