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
                                          float* __restrict__ base32, const float* __restrict__ base_in) {
  __shared__ float arow[kMaxRank];
  const long long row = blockIdx.x;  // h*I + i
  const int h = (int)(row / I);
  if (threadIdx.x < R) arow[threadIdx.x] = A ? A[row * R + threadIdx.x] : 0.f;
  __syncthreads();
  const float g = gain ? gain[0] : 1.0f;
  const float* Bh = Bm ? Bm + (size_t)h * R * O : nullptr;
  for (int o = threadIdx.x; o < O; o += blockDim.x) {
    const long long idx = row * O + o;
    const float w = base_in ? base_in[idx] : scaffold_value(key, (uint64_t)idx, stdv, dist);
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

// Adapter gradients from the dense projection gradient dW [Hm, I, O] (fp32), one pass:
//   dA[h,i,:] = s * sum_o dW[h,i,o] B[h,:,o]     dB[h,:,o] = s * sum_i A[h,i,:] dW[h,i,o]
//   dgain     = sum dW * W_seed                   (W_seed regenerated, or read from base32)
// Block (h, row chunk rc of RI rows, column chunk cc of 256 columns); thread t owns
// column o = 256 cc + t. dB partials over the block's rows stay in registers; dA partials
// over the block's columns are reduced warp by warp (shuffles) and then across the 8
// warps in shared memory. Partials go to fixed slots (no atomics) and
// scaffold_sum_partials adds them in a fixed order, so the result is bitwise
// reproducible.
constexpr int kAdRows = 32;

template <int R>
__global__ void __launch_bounds__(256) scaffold_adapter_grad_kernel(
    uint64_t key, float stdv, int dist, int I, int O, const float* __restrict__ dW, const float* __restrict__ A,
    const float* __restrict__ Bm, const float* __restrict__ base32, float* __restrict__ dA_part,
    float* __restrict__ dB_part, float* __restrict__ gain_part, int want_gain) {
  const int cc = blockIdx.x, rc = blockIdx.y, h = blockIdx.z;
  const int n_cc = gridDim.x, n_rc = gridDim.y;
  const int t = threadIdx.x, lane = t % 32, warp = t / 32;
  const int o = cc * 256 + t;
  const int i0 = rc * kAdRows;
  __shared__ float sA[kAdRows][R];
  __shared__ float sdA[8][kAdRows][R];
  for (int k = t; k < kAdRows * R; k += 256) {
    const int ii = i0 + k / R;
    sA[k / R][k % R] = ii < I ? A[((size_t)h * I + ii) * R + k % R] : 0.f;
  }
  float b[R];
#pragma unroll
  for (int r = 0; r < R; ++r) b[r] = o < O ? Bm[((size_t)h * R + r) * O + o] : 0.f;
  __syncthreads();
  float accB[R];
#pragma unroll
  for (int r = 0; r < R; ++r) accB[r] = 0.f;
  float g = 0.f;
  for (int ii = 0; ii < kAdRows; ++ii) {
    const int i = i0 + ii;
    float w = 0.f;
    const size_t idx = ((size_t)h * I + i) * O + o;
    if (i < I && o < O) {
      w = dW[idx];
      if (want_gain) {
        const float base = base32 ? base32[idx] : scaffold_value(key, (uint64_t)idx, stdv, dist);
        g += w * base;
      }
    }
#pragma unroll
    for (int r = 0; r < R; ++r) accB[r] += sA[ii][r] * w;
#pragma unroll
    for (int r = 0; r < R; ++r) {
      float q = w * b[r];
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) q += __shfl_xor_sync(0xffffffffu, q, off);
      if (lane == 0) sdA[warp][ii][r] = q;
    }
  }
  // dB partial of this row chunk: [h, rc, r, o]
  if (o < O)
#pragma unroll
    for (int r = 0; r < R; ++r) dB_part[(((size_t)h * n_rc + rc) * R + r) * O + o] = accB[r];
  __syncthreads();
  // dA partial of this column chunk: [h, cc, i, r] (warps summed in a fixed order)
  for (int k = t; k < kAdRows * R; k += 256) {
    const int ii = k / R, r = k % R;
    if (i0 + ii >= I) continue;
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) s += sdA[w][ii][r];
    dA_part[(((size_t)h * n_cc + cc) * I + i0 + ii) * R + r] = s;
  }
  if (want_gain) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) g += __shfl_xor_sync(0xffffffffu, g, off);
    __shared__ float sg[8];
    if (lane == 0) sg[warp] = g;
    __syncthreads();
    if (t == 0) {
      float s = 0.f;
      for (int w = 0; w < 8; ++w) s += sg[w];
      gain_part[((size_t)h * n_rc + rc) * n_cc + cc] = s;
    }
  }
}

// out[j] = scale * sum_{c < C} part[(g * C + c) * J + j] for j < J, g < G (out [G, J]).
__global__ void scaffold_sum_partials_kernel(const float* __restrict__ part, int G, int C, long long J, float scale,
                                             float* __restrict__ out) {
  const long long n = (long long)G * J;
  for (long long k = (long long)blockIdx.x * blockDim.x + threadIdx.x; k < n; k += (long long)gridDim.x * blockDim.x) {
    const long long gi = k / J, j = k % J;
    float s = 0.f;
    for (int c = 0; c < C; ++c) s += part[(gi * C + c) * J + j];
    out[k] = scale * s;
  }
}

template <typename T>
T* opt(const c10::optional<at::Tensor>& t) {
  return t ? reinterpret_cast<T*>(t->data_ptr()) : nullptr;
}

}  // namespace

// rows = H*I; A [H*I, R] fp32 (or None), B [H, R, O] fp32 (or None), gain [1] (or None);
// base_in: the cached fp32 W_seed (or None: regenerate it from the seed).
void scaffold_effective(int64_t key, double stdv, int64_t dist, int64_t rows, int64_t I, int64_t O, int64_t R,
                        const c10::optional<at::Tensor>& A, const c10::optional<at::Tensor>& B,
                        const c10::optional<at::Tensor>& gain, double scale, const c10::optional<at::Tensor>& out16,
                        const c10::optional<at::Tensor>& out32, const c10::optional<at::Tensor>& base32,
                        const c10::optional<at::Tensor>& base_in) {
  TORCH_CHECK(R <= kMaxRank, "scaffold rank must be <= 64");
  const at::Tensor& any = out16 ? *out16 : (out32 ? *out32 : *base32);
  c10::cuda::CUDAGuard g(any.get_device());
  auto st = at::cuda::getCurrentCUDAStream(any.get_device()).stream();
  scaffold_effective_kernel<<<(unsigned)rows, 256, 0, st>>>((uint64_t)key, (float)stdv, (int)dist, (int)I, (int)O,
                                                            (int)R, opt<const float>(A), opt<const float>(B),
                                                            opt<const float>(gain), (float)scale,
                                                            opt<__nv_bfloat16>(out16), opt<float>(out32),
                                                            opt<float>(base32), opt<const float>(base_in));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Adapter gradients of one scaffolded projection from its dense gradient dW [Hm, I, O]:
// dA [Hm, I, R] and dB [Hm, R, O] (scaled by `scale`), and, with `gain_out`, the gain
// gradient sum(dW * W_seed) written (not added) to gain_out[0]. `base32`: the cached
// fp32 W_seed, or None to regenerate it from (key, stdv, dist). `work`: fp32 scratch of
// at least scaffold_adapter_work(Hm, I, O, R) elements.
void scaffold_adapter_grad(int64_t key, double stdv, int64_t dist, int64_t Hm, int64_t I, int64_t O, int64_t R,
                           const at::Tensor& dW, const at::Tensor& A, const at::Tensor& B,
                           const c10::optional<at::Tensor>& base32, double scale, const at::Tensor& dA,
                           const at::Tensor& dB, const c10::optional<at::Tensor>& gain_out, const at::Tensor& work) {
  TORCH_CHECK(R == 4 || R == 8 || R == 16 || R == 32, "adapter rank 4, 8, 16 or 32 on the fused path");
  TORCH_CHECK(dW.scalar_type() == at::kFloat && dW.is_contiguous() && dW.numel() == Hm * I * O, "dW [Hm, I, O] fp32");
  TORCH_CHECK(A.is_contiguous() && B.is_contiguous() && A.numel() == Hm * I * R && B.numel() == Hm * R * O,
              "A [Hm, I, R], B [Hm, R, O] contiguous fp32");
  const int n_cc = (int)((O + 255) / 256), n_rc = (int)((I + kAdRows - 1) / kAdRows);
  const long long nA = Hm * n_cc * I * R, nB = Hm * n_rc * R * O, nG = Hm * n_rc * n_cc;
  TORCH_CHECK(work.numel() >= nA + nB + nG, "scaffold_adapter_grad: work buffer too small");
  c10::cuda::CUDAGuard g(dW.get_device());
  auto st = at::cuda::getCurrentCUDAStream(dW.get_device()).stream();
  float* pa = work.data_ptr<float>();
  float* pb = pa + nA;
  float* pg = pb + nB;
  dim3 grid(n_cc, n_rc, (unsigned)Hm);
  const float* b32 = base32 ? base32->data_ptr<float>() : nullptr;
  const int want = gain_out ? 1 : 0;
#define BD_AD(RR)                                                                                                   \
  scaffold_adapter_grad_kernel<RR><<<grid, 256, 0, st>>>((uint64_t)key, (float)stdv, (int)dist, (int)I, (int)O,    \
                                                         dW.data_ptr<float>(), A.data_ptr<float>(),                \
                                                         B.data_ptr<float>(), b32, pa, pb, pg, want)
  switch (R) {
    case 4: BD_AD(4); break;
    case 8: BD_AD(8); break;
    case 16: BD_AD(16); break;
    default: BD_AD(32); break;
  }
#undef BD_AD
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  scaffold_sum_partials_kernel<<<148 * 2, 256, 0, st>>>(pa, (int)Hm, n_cc, I * R, (float)scale, dA.data_ptr<float>());
  scaffold_sum_partials_kernel<<<148 * 2, 256, 0, st>>>(pb, (int)Hm, n_rc, R * O, (float)scale, dB.data_ptr<float>());
  if (gain_out)
    scaffold_sum_partials_kernel<<<1, 256, 0, st>>>(pg, 1, (int)nG, 1, 1.0f, gain_out->data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

int64_t scaffold_adapter_work(int64_t Hm, int64_t I, int64_t O, int64_t R) {
  const int64_t n_cc = (O + 255) / 256, n_rc = (I + kAdRows - 1) / kAdRows;
  return Hm * n_cc * I * R + Hm * n_rc * R * O + Hm * n_rc * n_cc;
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
