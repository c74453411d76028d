// decode.cu — one-token recurrent attention step for generation.
//
// For each (b, h): a[b,h,:] = rho[b,h]^T q[b,h,:]   (read BEFORE the update)
//                  rho[b,h] <- (rho[b,h] + q[b,h,:] (x) v[b,:]) * gamma_h
// (burn_dragon_core/src/model/sequence/linear.rs:18-60 with T = 1). The state is the
// whole cost of a decode token: it is read and written at most once here, in place, and
// without decay only the rows whose q is nonzero are touched.
// Grid: (row chunks of Nh, B*H); 256 threads = 64 column groups of 4 floats x 4 row
// phases; the 4 phases reduce through smem and one atomicAdd per column lands in `a`
// (which the caller zeroes).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_bf16.h>
#include <torch/extension.h>

#include <type_traits>

namespace bd {
namespace {

constexpr int kRows = 64;  // latent rows per CTA

__device__ __forceinline__ float to_f(float x) { return x; }
__device__ __forceinline__ float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }

// 4 state values: fp32 (16 bytes) or bf16 (8 bytes, rounded to nearest on store)
__device__ __forceinline__ float4 ld4(const float* p) { return *reinterpret_cast<const float4*>(p); }
__device__ __forceinline__ float4 ld4(const __nv_bfloat16* p) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
  const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
  return make_float4(a.x, a.y, b.x, b.y);
}
__device__ __forceinline__ void st4(float* p, float4 v) { *reinterpret_cast<float4*>(p) = v; }
__device__ __forceinline__ void st4(__nv_bfloat16* p, float4 v) {
  __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.y), b = __floats2bfloat162_rn(v.z, v.w);
  uint2 u;
  u.x = *reinterpret_cast<unsigned int*>(&a);
  u.y = *reinterpret_cast<unsigned int*>(&b);
  *reinterpret_cast<uint2*>(p) = u;
}

template <typename QT, typename RT>
__global__ void rho_step_kernel(RT* __restrict__ rho, const QT* __restrict__ q, long long q_row_stride,
                                const float* __restrict__ v, const float* __restrict__ gamma, float* __restrict__ a,
                                int H, int Nh, int D) {
  __shared__ float4 red[4][64];
  const int bh = blockIdx.y;
  const int b = bh / H, h = bh % H;
  const int j0 = blockIdx.x * kRows;
  const int c4 = threadIdx.x & 63;  // column group (4 floats)
  const int ph = threadIdx.x >> 6;  // row phase 0..3
  const float g = gamma ? gamma[h] : 1.0f;
  RT* R = rho + ((size_t)bh * Nh) * D;
  const QT* qb = q + (size_t)b * q_row_stride + (size_t)h * Nh;
  float4 vv = make_float4(0.f, 0.f, 0.f, 0.f);
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  const int D4 = D / 4;
  for (int cb = 0; cb < D4; cb += 64) {
    const int c = cb + c4;
    const bool on = c < D4;
    acc = make_float4(0.f, 0.f, 0.f, 0.f);
    if (on) {
      vv = reinterpret_cast<const float4*>(v + (size_t)b * D)[c];
      for (int j = j0 + ph; j < min(j0 + kRows, Nh); j += 4) {
        const float qj = to_f(qb[j]);
        // a latent row whose q is 0 neither changes rho (without decay) nor adds to a: its
        // read and write are skipped (exact; q is ReLU-sparse, so many rows are 0). The
        // branch is uniform over a warp (all its lanes share the row phase).
        if (qj == 0.0f && g == 1.0f) continue;
        float4 r = ld4(R + ((size_t)j * D4 + c) * 4);
        acc.x += qj * r.x;
        acc.y += qj * r.y;
        acc.z += qj * r.z;
        acc.w += qj * r.w;
        r.x = (r.x + qj * vv.x) * g;
        r.y = (r.y + qj * vv.y) * g;
        r.z = (r.z + qj * vv.z) * g;
        r.w = (r.w + qj * vv.w) * g;
        st4(R + ((size_t)j * D4 + c) * 4, r);
      }
    }
    red[ph][c4] = acc;
    __syncthreads();
    if (ph == 0 && on) {
      float4 s = red[0][c4];
#pragma unroll
      for (int k = 1; k < 4; ++k) {
        s.x += red[k][c4].x;
        s.y += red[k][c4].y;
        s.z += red[k][c4].z;
        s.w += red[k][c4].w;
      }
      float* dst = a + (size_t)bh * D + 4 * c;
      atomicAdd(dst + 0, s.x);
      atomicAdd(dst + 1, s.y);
      atomicAdd(dst + 2, s.z);
      atomicAdd(dst + 3, s.w);
    }
    __syncthreads();
  }
}

}  // namespace

// rho [B,H,Nh,D] fp32 or bf16 (updated in place); q rows [B, >= H*Nh] (bf16 or fp32, row stride
// q_row_stride elements); v [B,D] fp32; gamma [H] or None; a [B,H,D] fp32, pre-zeroed.
void rho_step(const at::Tensor& rho, const at::Tensor& q, int64_t q_row_stride, const at::Tensor& v,
              const c10::optional<at::Tensor>& gamma, const at::Tensor& a, int64_t B, int64_t H, int64_t Nh,
              int64_t D) {
  c10::cuda::CUDAGuard g(rho.get_device());
  TORCH_CHECK((rho.scalar_type() == at::kFloat || rho.scalar_type() == at::kBFloat16) &&
                  v.scalar_type() == at::kFloat && a.scalar_type() == at::kFloat,
              "rho_step: rho fp32 or bf16, v and a fp32");
  TORCH_CHECK(D % 4 == 0, "rho_step: D must be a multiple of 4");
  dim3 grid((unsigned)((Nh + kRows - 1) / kRows), (unsigned)(B * H));
  auto st = at::cuda::getCurrentCUDAStream(rho.get_device()).stream();
  const float* gp = gamma ? gamma->data_ptr<float>() : nullptr;
  TORCH_CHECK(q.scalar_type() == at::kBFloat16 || q.scalar_type() == at::kFloat, "rho_step: q must be bf16 or fp32");
  auto go = [&](auto* r) {
    using RT = std::remove_pointer_t<decltype(r)>;
    if (q.scalar_type() == at::kBFloat16)
      rho_step_kernel<__nv_bfloat16, RT><<<grid, 256, 0, st>>>(
          r, reinterpret_cast<const __nv_bfloat16*>(q.data_ptr()), q_row_stride, v.data_ptr<float>(), gp,
          a.data_ptr<float>(), (int)H, (int)Nh, (int)D);
    else
      rho_step_kernel<float, RT><<<grid, 256, 0, st>>>(r, q.data_ptr<float>(), q_row_stride, v.data_ptr<float>(), gp,
                                                       a.data_ptr<float>(), (int)H, (int)Nh, (int)D);
  };
  if (rho.scalar_type() == at::kFloat)
    go(rho.data_ptr<float>());
  else
    go(reinterpret_cast<__nv_bfloat16*>(rho.data_ptr()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace bd
