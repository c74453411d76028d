// gemm_inst_c.cu — the fused BDH epilogues (ReLU+RoPE, causal scores, gate,
// decoder backward, dQ).
#include "gemm_launch.cuh"
namespace bd {
const Entry kGemmTableC[] = {
    BD_ENTRY(128, false, true, EPI_RELU_ROPE), BD_ENTRY(128, false, false, EPI_SCORES),
    BD_ENTRY(256, false, false, EPI_SCORES),   BD_ENTRY(64, false, false, EPI_SCORES),
    BD_ENTRY(128, false, true, EPI_GATE),      BD_ENTRY(128, false, false, EPI_DEC_BWD),
    BD_ENTRY(128, false, true, EPI_DQ),        BD_ENTRY(128, false, false, EPI_DQ),
};
const int kGemmTableCSize = sizeof(kGemmTableC) / sizeof(Entry);
}  // namespace bd
