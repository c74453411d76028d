// gdpo.cu — per-row percentile thresholds for GDPO advantage gating
// (burn_dragon_train/src/train/gdpo/cubecl.rs:181-279): for each row of a [rows, group]
// matrix, the linearly interpolated quantile q of the row (NaN read as 0, +-inf clamped
// to +-FLT_MAX). One block per row sorts the row in shared memory with a bitonic
// network (padded with +inf to a power of two, group <= 1024) instead of the
// reference's per-thread insertion sort.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <cfloat>

namespace bd {
namespace {

__global__ void percentile_kernel(const float* __restrict__ v, long long row_stride, int group, float q,
                                  float* __restrict__ out) {
  __shared__ float s[1024];
  const int row = blockIdx.x;
  int n = 1;
  while (n < group) n <<= 1;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    float x = INFINITY;
    if (i < group) {
      x = v[(size_t)row * row_stride + i];
      if (isnan(x)) x = 0.f;
      if (isinf(x)) x = x < 0.f ? -FLT_MAX : FLT_MAX;
    }
    s[i] = x;
  }
  __syncthreads();
  for (int k = 2; k <= n; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const int l = i ^ j;
        if (l > i) {
          const bool up = (i & k) == 0;
          const float a = s[i], b = s[l];
          if ((a > b) == up) {
            s[i] = b;
            s[l] = a;
          }
        }
      }
      __syncthreads();
    }
  }
  if (threadIdx.x == 0) {
    const float pos = (float)(group - 1) * q;
    const int lo = (int)pos;
    const int hi = lo + 1 < group ? lo + 1 : lo;
    const float w = pos - (float)lo;
    out[row] = s[lo] + (s[hi] - s[lo]) * w;
  }
}

}  // namespace

void percentile_thresholds(const at::Tensor& values, double q, const at::Tensor& out) {
  c10::cuda::CUDAGuard g(values.get_device());
  TORCH_CHECK(values.dim() == 2 && values.scalar_type() == at::kFloat, "values must be [rows, group] fp32");
  TORCH_CHECK(values.stride(1) == 1, "values rows must be contiguous");
  const int group = (int)values.size(1);
  TORCH_CHECK(group >= 1 && group <= 1024, "group size must be in [1, 1024]");
  const int rows = (int)values.size(0);
  if (rows == 0) return;
  percentile_kernel<<<rows, 256, 0, at::cuda::getCurrentCUDAStream(values.get_device()).stream()>>>(
      values.data_ptr<float>(), values.stride(0), group, (float)q, out.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace bd
