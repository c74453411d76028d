// gemm_table.h — the instantiation table of the tcgen05 GEMM engine. The kernel
// template is instantiated in five translation units (gemm_inst_{a..e}.cu) so nvcc
// compiles them in parallel; gemm_host.cu looks a launch function up by its
// (tile N, A major, B major, epilogue) key.
#pragma once
#include <cuda_runtime.h>

namespace bd {

struct GemmParams;
using LaunchFn = void (*)(const GemmParams&, cudaStream_t, int);

struct Entry {
  int bn;
  bool a_mn, b_mn;
  int epi;
  LaunchFn fn;
  bool pair = false;  // 2-CTA (cta_group::2) kernel: 256-row tiles on a CTA pair
};

int num_sms_of(int dev);

extern const Entry kGemmTableA[];
extern const int kGemmTableASize;
extern const Entry kGemmTableB[];
extern const int kGemmTableBSize;
extern const Entry kGemmTableC[];
extern const int kGemmTableCSize;
extern const Entry kGemmTableD[];
extern const int kGemmTableDSize;
extern const Entry kGemmTableE[];
extern const int kGemmTableESize;

}  // namespace bd
