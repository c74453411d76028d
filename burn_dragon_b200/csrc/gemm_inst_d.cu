// gemm_inst_d.cu — CTA-pair (cta_group::2) instantiations for the MMA-bound contractions.
#include "gemm_launch.cuh"
namespace bd {
const Entry kGemmTableD[] = {
    BD_PAIR(256, true, true, EPI_F32),     // weight gradients, dV, d(lm_head)
    BD_PAIR(256, false, true, EPI_F32),    // decoder product, S V, logits
    BD_PAIR(256, false, false, EPI_F32),   // d(an), per-head dv, dC V^T
    BD_PAIR(128, false, false, EPI_F32),
    BD_PAIR(256, false, false, EPI_SCORES),
    BD_PAIR(128, false, false, EPI_SCORES),
};
const int kGemmTableDSize = sizeof(kGemmTableD) / sizeof(Entry);
}  // namespace bd
