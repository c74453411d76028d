// gemm_launch.cuh — launch helper shared by the GEMM instantiation units.
#pragma once
#include <c10/cuda/CUDAException.h>

#include <algorithm>

#include "gemm_sm100.cuh"
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

#define BD_ENTRY(BN, AMN, BMN, EPI) Entry{BN, AMN, BMN, EPI, &launch_one<BN, AMN, BMN, EPI>}

}  // namespace bd
