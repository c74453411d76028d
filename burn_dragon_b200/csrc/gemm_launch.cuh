// gemm_launch.cuh — launch helper shared by the GEMM instantiation units.
#pragma once
#include <c10/cuda/CUDAException.h>

#include <algorithm>

#include "gemm_sm100.cuh"
#include "gemm_sm100_2cta.cuh"
#include "gemm_table.h"

namespace bd {

template <int BN, bool A_MN, bool B_MN, int EPI>
void launch_one(const GemmParams& p, cudaStream_t stream, int dev) {
  using Cfg = GemmCfg<BN, epi_kind<EPI>()>;
  auto kern = gemm_sm100_kernel<BN, A_MN, B_MN, EPI>;
  static bool attr_set[64] = {false};
  if (!attr_set[dev]) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM));
    attr_set[dev] = true;
  }
  const long long total = (long long)p.tiles_m * p.tiles_n * p.splits * p.Z1 * p.Z2;
  const int grid = (int)std::min<long long>(total, num_sms_of(dev));
  kern<<<grid, Cfg::THREADS, Cfg::SMEM, stream>>>(p);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

#define BD_ENTRY(BN, AMN, BMN, EPI) Entry{BN, AMN, BMN, EPI, &launch_one<BN, AMN, BMN, EPI>, false}

// Launch of the CTA-pair kernel: clusters of 2, one pair per two SMs (persistent).
template <int BN, bool A_MN, bool B_MN, int EPI>
void launch_pair(const GemmParams& p, cudaStream_t stream, int dev) {
  using Cfg = Gemm2Cfg<BN, epi_kind<EPI>()>;
  auto kern = gemm_sm100_2cta_kernel<BN, A_MN, B_MN, EPI>;
  static bool attr_set[64] = {false};
  if (!attr_set[dev]) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM));
    attr_set[dev] = true;
  }
  const long long total = (long long)p.tiles_m * p.tiles_n * p.splits * p.Z1 * p.Z2;
  const int clusters = (int)std::min<long long>(total, num_sms_of(dev) / 2);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(2 * clusters), 1, 1);
  cfg.blockDim = dim3(Cfg::THREADS, 1, 1);
  cfg.dynamicSmemBytes = Cfg::SMEM;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  C10_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kern, p));
}

#define BD_PAIR(BN, AMN, BMN, EPI) Entry{BN, AMN, BMN, EPI, &launch_pair<BN, AMN, BMN, EPI>, true}

}  // namespace bd
