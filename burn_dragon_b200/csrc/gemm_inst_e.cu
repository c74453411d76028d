// gemm_inst_e.cu — CTA-pair 256 x 256 tiles for the TMA-epilogue BDH modes (x-projection
// + RoPE, gate, decoder backward, dQ).
#include "gemm_launch.cuh"
namespace bd {
const Entry kGemmTableE[] = {
    BD_PAIR(256, false, true, EPI_RELU_ROPE),
    BD_PAIR(256, false, true, EPI_GATE),
    BD_PAIR(256, false, false, EPI_DEC_BWD),
    BD_PAIR(256, false, true, EPI_DQ),
};
const int kGemmTableESize = sizeof(kGemmTableE) / sizeof(Entry);
}  // namespace bd
