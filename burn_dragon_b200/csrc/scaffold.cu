// scaffold.cu — random-scaffold projections regenerated from the seed on the device.
//
// Generator contract "dragon-scaffold-v1" (this framework's; the reference's generator
// crate is not part of its repository):
//   key        = mix64(seed ^ fnv1a64(path))
//   u_k(idx)   = (mix64(key ^ mix64(12*idx + k + 1)) >> 40) * 2^-24      k = 0..11
//   gaussian_clt12: w = std * (sum_k u_k - 6)
//   rademacher    : w = std * (mix64(key ^ mix64(12*idx + 1)) >> 63 ? +1 : -1)
// with mix64 the SplitMix64 finalizer (Steele, Lea, Flood 2014). Every element is a pure
// function of (seed, path, flat index), so any kernel can regenerate any element.
//
// scaffold_effective: W_eff[h,i,o] = gain * W_seed[h,i,o] + scale * sum_r A[h,i,r] B[h,r,o]
// (burn_dragon_core/src/model/scaffold.rs:21-124 "effective"), written as the bf16 GEMM
// operand (and optionally fp32), without ever storing W_seed.
// scaffold_gain_grad: d(gain) = sum(dW_eff * W_seed), W_seed regenerated again.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_bf16.h>
#include <torch/extension.h>

namespace bd {
namespace {

__device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z ^= z >> 30;
  z *= 0xbf58476d1ce4e5b9ull;
  z ^= z >> 27;
  z *= 0x94d049bb133111ebull;
  z ^= z >> 31;
  return z;
}

__device__ __forceinline__ float scaffold_value(uint64_t key, uint64_t idx, float stdv, int dist) {
  if (dist == 1) {
    const uint64_t h = mix64(key ^ mix64(12ull * idx + 1ull));
    return (h >> 63) ? stdv : -stdv;
  }
  float s = 0.f;
#pragma unroll
  for (int k = 0; k < 12; ++k) {
    const uint64_t h = mix64(key ^ mix64(12ull * idx + (uint64_t)k + 1ull));
    s += (float)(h >> 40) * (1.0f / 16777216.0f);
  }
  return stdv * (s - 6.0f);
}

constexpr int kMaxRank = 64;

// One block per (h, i) row; threads over o.
__global__ void scaffold_effective_kernel(uint64_t key, float stdv, int dist, int I, int O, int R,
                                          const float* __restrict__ A, const float* __restrict__ Bm,
                                          const float* __restrict__ gain, float scale,
                                          __nv_bfloat16* __restrict__ out16, float* __restrict__ out32,
                                          float* __restrict__ base32) {
  __shared__ float arow[kMaxRank];
  const long long row = blockIdx.x;  // h*I + i
  const int h = (int)(row / I);
  if (threadIdx.x < R) arow[threadIdx.x] = A ? A[row * R + threadIdx.x] : 0.f;
  __syncthreads();
  const float g = gain ? gain[0] : 1.0f;
  const float* Bh = Bm ? Bm + (size_t)h * R * O : nullptr;
  for (int o = threadIdx.x; o < O; o += blockDim.x) {
    const long long idx = row * O + o;
    const float w = scaffold_value(key, (uint64_t)idx, stdv, dist);
    float acc = 0.f;
    if (Bh)
      for (int r = 0; r < R; ++r) acc += arow[r] * Bh[(size_t)r * O + o];
    const float y = g * w + scale * acc;
    if (out16) out16[idx] = __float2bfloat16_rn(y);
    if (out32) out32[idx] = y;
    if (base32) base32[idx] = w;
  }
}

__global__ void scaffold_gain_grad_kernel(uint64_t key, float stdv, int dist, long long n,
                                          const float* __restrict__ dW, float* __restrict__ out) {
  float s = 0.f;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    s += dW[i] * scaffold_value(key, (uint64_t)i, stdv, dist);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  __shared__ float sh[32];
  if (threadIdx.x % 32 == 0) sh[threadIdx.x / 32] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < blockDim.x / 32 ? sh[threadIdx.x] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (threadIdx.x == 0) atomicAdd(out, t);
  }
}

template <typename T>
T* opt(const c10::optional<at::Tensor>& t) {
  return t ? reinterpret_cast<T*>(t->data_ptr()) : nullptr;
}

}  // namespace

// rows = H*I; A [H*I, R] fp32 (or None), B [H, R, O] fp32 (or None), gain [1] (or None).
void scaffold_effective(int64_t key, double stdv, int64_t dist, int64_t rows, int64_t I, int64_t O, int64_t R,
                        const c10::optional<at::Tensor>& A, const c10::optional<at::Tensor>& B,
                        const c10::optional<at::Tensor>& gain, double scale, const c10::optional<at::Tensor>& out16,
                        const c10::optional<at::Tensor>& out32, const c10::optional<at::Tensor>& base32) {
  TORCH_CHECK(R <= kMaxRank, "scaffold rank must be <= 64");
  const at::Tensor& any = out16 ? *out16 : (out32 ? *out32 : *base32);
  c10::cuda::CUDAGuard g(any.get_device());
  auto st = at::cuda::getCurrentCUDAStream(any.get_device()).stream();
  scaffold_effective_kernel<<<(unsigned)rows, 256, 0, st>>>((uint64_t)key, (float)stdv, (int)dist, (int)I, (int)O,
                                                            (int)R, opt<const float>(A), opt<const float>(B),
                                                            opt<const float>(gain), (float)scale,
                                                            opt<__nv_bfloat16>(out16), opt<float>(out32),
                                                            opt<float>(base32));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// out[0] += sum(dW * W_seed)
void scaffold_gain_grad(int64_t key, double stdv, int64_t dist, const at::Tensor& dW, const at::Tensor& out) {
  c10::cuda::CUDAGuard g(dW.get_device());
  auto st = at::cuda::getCurrentCUDAStream(dW.get_device()).stream();
  scaffold_gain_grad_kernel<<<148 * 4, 256, 0, st>>>((uint64_t)key, (float)stdv, (int)dist, dW.numel(),
                                                     dW.data_ptr<float>(), out.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace bd
