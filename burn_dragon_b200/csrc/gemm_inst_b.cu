// gemm_inst_b.cu — fp32-output instantiations with MN-major operands (weight
// gradients, value products, split-K partials).
#include "gemm_launch.cuh"
namespace bd {
const Entry kGemmTableB[] = {
    BD_ENTRY(256, false, true, EPI_F32), BD_ENTRY(128, false, true, EPI_F32),
    BD_ENTRY(64, false, true, EPI_F32),  BD_ENTRY(256, true, true, EPI_F32),
    BD_ENTRY(128, true, true, EPI_F32),  BD_ENTRY(64, true, true, EPI_F32),
    BD_ENTRY(256, true, false, EPI_F32), BD_ENTRY(128, true, false, EPI_F32),
    BD_ENTRY(64, true, false, EPI_F32),
};
const int kGemmTableBSize = sizeof(kGemmTableB) / sizeof(Entry);
}  // namespace bd
