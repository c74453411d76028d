// gemm_inst_a.cu — plain bf16 / fp32 epilogue instantiations.
#include "gemm_launch.cuh"
namespace bd {
const Entry kGemmTableA[] = {
    BD_ENTRY(256, false, false, EPI_BF16), BD_ENTRY(128, false, false, EPI_BF16),
    BD_ENTRY(64, false, false, EPI_BF16),  BD_ENTRY(256, false, true, EPI_BF16),
    BD_ENTRY(64, false, true, EPI_BF16),   BD_ENTRY(128, false, true, EPI_BF16),   BD_ENTRY(256, false, false, EPI_F32),
    BD_ENTRY(128, false, false, EPI_F32),  BD_ENTRY(64, false, false, EPI_F32),
    // tensor-parallel decoder product with the reduce-scatter in the epilogue
    BD_ENTRY(256, false, true, EPI_F32_SCATTER), BD_ENTRY(128, false, true, EPI_F32_SCATTER),
    BD_ENTRY(64, false, true, EPI_F32_SCATTER),
};
const int kGemmTableASize = sizeof(kGemmTableA) / sizeof(Entry);
}  // namespace bd
