// gemm_host.cu — host side of the tcgen05 GEMM engine: TMA tensor-map encoding,
// tile-grid sizing for a persistent launch over all SMs, and the instantiation table.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cudaTypedefs.h>
#include <torch/extension.h>

#include <cstdlib>
#include <mutex>
#include <stdexcept>
#include <string>
#include <vector>

#include "gemm_sm100.cuh"
#include "gemm_table.h"

namespace bd {

namespace {

PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t st = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q);
    TORCH_CHECK(st == cudaSuccess && q == cudaDriverEntryPointSuccess && ptr != nullptr,
                "burn_dragon_b200: cuTensorMapEncodeTiled is unavailable");
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

// Operand geometry, in elements: a 4-D view (inner, outer, z1, z2) of bf16 memory.
struct Geom {
  int64_t inner, outer, outer_stride, z1c, z1s, z2c, z2s;
  bool use_z1, use_z2;
};

Geom parse_geom(const std::vector<int64_t>& g) {
  TORCH_CHECK(g.size() == 9, "operand geometry needs 9 entries");
  return Geom{g[0], g[1], g[2], g[3], g[4], g[5], g[6], g[7] != 0, g[8] != 0};
}

CUtensorMap encode_map(const at::Tensor& t, const Geom& g, uint32_t box_inner, uint32_t box_outer) {
  TORCH_CHECK(t.scalar_type() == at::kBFloat16, "GEMM operands must be bf16");
  TORCH_CHECK(t.is_cuda(), "GEMM operands must be CUDA tensors");
  const uintptr_t base = reinterpret_cast<uintptr_t>(t.data_ptr());
  TORCH_CHECK(base % 16 == 0, "GEMM operand base must be 16-byte aligned");
  auto chk16 = [](int64_t elems) {
    TORCH_CHECK((elems * 2) % 16 == 0, "GEMM operand strides must be multiples of 16 bytes");
  };
  chk16(g.outer_stride);
  TORCH_CHECK(g.inner % 8 == 0, "GEMM operand inner extent must be a multiple of 8 elements");
  cuuint64_t dims[4] = {(cuuint64_t)g.inner, (cuuint64_t)g.outer, (cuuint64_t)(g.use_z1 ? g.z1c : 1),
                        (cuuint64_t)(g.use_z2 ? g.z2c : 1)};
  const int64_t fallback = ((g.outer * g.outer_stride * 2 + 15) / 16) * 16;
  const int64_t s1 = g.outer_stride * 2;
  const int64_t s2 = g.use_z1 ? g.z1s * 2 : fallback;
  const int64_t s3 = g.use_z2 ? g.z2s * 2 : fallback;
  if (g.use_z1) chk16(g.z1s);
  if (g.use_z2) chk16(g.z2s);
  cuuint64_t strides[3] = {(cuuint64_t)s1, (cuuint64_t)s2, (cuuint64_t)s3};
  cuuint32_t box[4] = {box_inner, box_outer, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUtensorMap m;
  CUresult r = get_encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, t.data_ptr(), dims, strides, box,
                               estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed with code ", (int)r);
  return m;
}

// 32-row box map over an output-shaped bf16 matrix (cols, rows, z1, z2) for the TMA
// epilogue, `cols` = 64 (128-byte swizzle) or 32 (64-byte swizzle); strides in elements.
CUtensorMap encode_out_map(const void* ptr, int64_t N, int64_t M, int64_t ld, int64_t Z1, int64_t sz1, int64_t Z2,
                           int64_t sz2, uint32_t cols) {
  TORCH_CHECK(reinterpret_cast<uintptr_t>(ptr) % 16 == 0, "TMA epilogue tensors must be 16-byte aligned");
  const int64_t fallback = ((M * ld * 2 + 15) / 16) * 16;
  cuuint64_t dims[4] = {(cuuint64_t)N, (cuuint64_t)M, (cuuint64_t)Z1, (cuuint64_t)Z2};
  cuuint64_t strides[3] = {(cuuint64_t)(ld * 2), (cuuint64_t)(Z1 > 1 ? sz1 * 2 : fallback),
                           (cuuint64_t)(Z2 > 1 ? sz2 * 2 : fallback)};
  cuuint32_t box[4] = {cols, 32, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUtensorMap m;
  CUresult r = get_encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(ptr), dims, strides, box,
                               estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                               cols == 32 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (epilogue map) failed with code ", (int)r);
  return m;
}

// The RoPE phase table [T, Nh/2] of half2 (cos, sin) words as 32-row boxes of cols / 2
// words: the byte geometry (and swizzle) of a 32 x cols bf16 output box, so chunk c of a
// table box holds the phases of chunk c of the x / q boxes.
CUtensorMap encode_table_map(const void* ptr, int64_t pairs, int64_t T, uint32_t cols) {
  TORCH_CHECK(reinterpret_cast<uintptr_t>(ptr) % 16 == 0, "RoPE table must be 16-byte aligned");
  cuuint64_t dims[4] = {(cuuint64_t)pairs, (cuuint64_t)T, 1, 1};
  const cuuint64_t row = (cuuint64_t)pairs * 4;
  cuuint64_t strides[3] = {row, row * (cuuint64_t)T, row * (cuuint64_t)T};
  cuuint32_t box[4] = {cols / 2, 32, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUtensorMap m;
  CUresult r = get_encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_INT32, 4, const_cast<void*>(ptr), dims, strides, box, estr,
                               CU_TENSOR_MAP_INTERLEAVE_NONE,
                               cols == 32 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (RoPE table map) failed with code ", (int)r);
  return m;
}

int num_sms(int dev) {
  static int cached[64] = {0};
  if (cached[dev] == 0) {
    int n = 0;
    C10_CUDA_CHECK(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
    cached[dev] = n;
  }
  return cached[dev];
}

}  // namespace

int num_sms_of(int dev) { return num_sms(dev); }

namespace {
const Entry* find_entry(int bn, bool a_mn, bool b_mn, int epi, bool pair) {
  const Entry* tables[5] = {kGemmTableA, kGemmTableB, kGemmTableC, kGemmTableD, kGemmTableE};
  const int sizes[5] = {kGemmTableASize, kGemmTableBSize, kGemmTableCSize, kGemmTableDSize, kGemmTableESize};
  for (int t = 0; t < 5; ++t)
    for (int i = 0; i < sizes[t]; ++i) {
      const Entry& en = tables[t][i];
      if (en.bn == bn && en.a_mn == a_mn && en.b_mn == b_mn && en.epi == epi && en.pair == pair) return &en;
    }
  return nullptr;
}
}  // namespace

// Generic entry: C[z1,z2] = epilogue(A[z1,z2] (M x K) * B[z1,z2]^T (N x K)).
void gemm(int64_t epi, int64_t bn, const at::Tensor& a, bool a_mn, std::vector<int64_t> a_geom,
          const at::Tensor& b, bool b_mn, std::vector<int64_t> b_geom, int64_t M, int64_t N, int64_t K,
          int64_t Z1, int64_t Z2, int64_t splits, bool causal_skip, const at::Tensor& out0,
          const c10::optional<at::Tensor>& out1, const c10::optional<at::Tensor>& aux0,
          const c10::optional<at::Tensor>& aux1, int64_t ld, int64_t sz1, int64_t sz2, int64_t split_stride,
          double alpha, double thr, const c10::optional<at::Tensor>& freq,
          const c10::optional<at::Tensor>& log2_decay, int64_t T, int64_t pos0, int64_t Nh,
          bool accumulate, bool row_decay, int64_t pair, const at::Tensor& err,
          const c10::optional<std::vector<int64_t>>& scatter, const c10::optional<at::Tensor>& acc_src,
          int64_t src_decay_T, const c10::optional<at::Tensor>& rope_tab) {
  // pair: 0 = 1-CTA kernel, 1 = CTA-pair kernel when instantiated and M >= 256
  const Entry* hit = nullptr;
  if (pair && M >= 256) hit = find_entry((int)bn, a_mn, b_mn, (int)epi, true);
  if (hit == nullptr) hit = find_entry((int)bn, a_mn, b_mn, (int)epi, false);
  if (hit == nullptr) {
    throw std::invalid_argument("burn_dragon_b200: no GEMM instantiation for bn=" + std::to_string(bn) +
                                " a_mn=" + std::to_string((int)a_mn) + " b_mn=" + std::to_string((int)b_mn) +
                                " epi=" + std::to_string(epi));
  }
  TORCH_CHECK(M > 0 && N > 0 && K > 0 && Z1 > 0 && Z2 > 0 && splits > 0, "bad GEMM sizes");
  TORCH_CHECK(N % 32 == 0, "GEMM N must be a multiple of 32");
  TORCH_CHECK(ld % 8 == 0 && sz1 % 8 == 0 && sz2 % 8 == 0 && split_stride % 8 == 0,
              "output strides must be multiples of 8 elements");
  TORCH_CHECK(err.scalar_type() == at::kInt && err.is_cuda(), "err must be an int32 CUDA tensor");
  const Geom ga = parse_geom(a_geom), gb = parse_geom(b_geom);
  const int dev = a.get_device();
  c10::cuda::CUDAGuard guard(dev);

  GemmParams p;
  memset(&p, 0, sizeof(p));
  p.ta = a_mn ? encode_map(a, ga, 64, 64) : encode_map(a, ga, 64, 128);
  // a CTA of a pair stages half of the B tile (BN/2 rows)
  p.tb = b_mn ? encode_map(b, gb, 64, 64) : encode_map(b, gb, 64, (uint32_t)(hit->pair ? bn / 2 : bn));
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.Z1 = (int)Z1;
  p.Z2 = (int)Z2;
  p.tiles_m = (int)((M + (hit->pair ? 255 : 127)) / (hit->pair ? 256 : 128));
  p.tiles_n = (int)((N + bn - 1) / bn);
  const int KB = (int)((K + 63) / 64);
  p.kb_per_split = (KB + (int)splits - 1) / (int)splits;
  p.splits = (KB + p.kb_per_split - 1) / p.kb_per_split;
  TORCH_CHECK(p.splits == splits, "split-K count ", splits, " does not fit ", KB, " K-blocks");
  p.a_z1 = ga.use_z1;
  p.a_z2 = ga.use_z2;
  p.b_z1 = gb.use_z1;
  p.b_z2 = gb.use_z2;
  p.causal_skip = causal_skip ? 1 : 0;
  p.err = err.data_ptr<int>();
  EpiParams& e = p.e;
  e.out0 = out0.data_ptr();
  e.out1 = out1 ? out1->data_ptr() : nullptr;
  e.aux0 = aux0 ? reinterpret_cast<const __nv_bfloat16*>(aux0->data_ptr()) : nullptr;
  e.aux1 = aux1 ? reinterpret_cast<const __nv_bfloat16*>(aux1->data_ptr()) : nullptr;
  e.ld = ld;
  e.sz1 = sz1;
  e.sz2 = sz2;
  e.split_stride = split_stride;
  e.alpha = (float)alpha;
  e.thr = (float)thr;
  e.freq = freq ? freq->data_ptr<float>() : nullptr;
  e.rope_tab = nullptr;
  e.rope_tma = 0;
  if (rope_tab && e.freq) {
    TORCH_CHECK(rope_tab->scalar_type() == at::kInt && rope_tab->numel() >= T * (Nh / 2) && Nh % 8 == 0,
                "rope_tab: int32 (half2) table of T x Nh/2 phases");
    if (epi == EPI_RELU_ROPE) {
      // staged by the epilogue's TMA ring (map encoded below with the output maps)
      TORCH_CHECK(T % 32 == 0 && Nh % 64 == 0 && rope_tab->is_contiguous(),
                  "staged RoPE table: T % 32 == 0, Nh % 64 == 0, contiguous");
      e.rope_tma = 1;
    } else {
      e.rope_tab = reinterpret_cast<const uint32_t*>(rope_tab->data_ptr());
    }
  }
  e.log2_decay = log2_decay ? log2_decay->data_ptr<float>() : nullptr;
  e.T = (int)T;
  e.pos0 = (int)pos0;
  e.Nh = (int)Nh;
  e.accumulate = accumulate ? 1 : 0;
  e.row_decay = row_decay ? 1 : 0;
  e.acc_src = acc_src ? acc_src->data_ptr<float>() : nullptr;
  e.src_decay_T = (int)src_decay_T;
  if (acc_src) {
    TORCH_CHECK(epi == EPI_F32 && accumulate && acc_src->scalar_type() == at::kFloat && splits == 1,
                "acc_src: fp32 source of an accumulating EPI_F32 GEMM without split-K");
    TORCH_CHECK(acc_src->numel() == out0.numel(), "acc_src must have out0's size and layout");
  }
  if (src_decay_T > 0) TORCH_CHECK(e.log2_decay != nullptr && acc_src, "src_decay_T needs log2_decay and acc_src");
  {
    static const int probe = [] {
      const char* v = std::getenv("BDH_GEMM_PROBE");
      return v ? std::atoi(v) : 0;
    }();
    e.probe = probe;
  }
  if (row_decay) TORCH_CHECK(e.log2_decay != nullptr, "row_decay needs log2_decay");
  if (epi == EPI_F32_SCATTER) {
    // scatter = [world, rows per owner, this rank, slot stride (elements), slot pointer per rank]
    TORCH_CHECK(scatter && scatter->size() >= 5, "EPI_F32_SCATTER needs the scatter description");
    const auto& sc = *scatter;
    const int64_t W = sc[0];
    TORCH_CHECK(W >= 1 && W <= 8 && (int64_t)sc.size() == 4 + W, "scatter: world in [1, 8], one pointer per rank");
    TORCH_CHECK(sc[1] > 0 && sc[1] * W >= M && Z1 == 1 && Z2 == 1 && splits == 1 && !causal_skip && !accumulate,
                "scatter: plain 2-D GEMM, rows covered by the owners");
    e.scatter_rows = (int)sc[1];
    e.scatter_rank = (int)sc[2];
    e.slot_stride = sc[3];
    for (int64_t r = 0; r < W; ++r) {
      e.peer[r] = reinterpret_cast<float*>(sc[4 + r]);
      TORCH_CHECK(sc[4 + r] % 16 == 0, "scatter slots must be 16-byte aligned");
    }
  } else if (epi == EPI_F32) {
    TORCH_CHECK(out0.scalar_type() == at::kFloat, "EPI_F32 output must be fp32");
    if (e.out1) TORCH_CHECK(out1->scalar_type() == at::kBFloat16, "EPI_F32 out1 (the copy) must be bf16");
  } else {
    TORCH_CHECK(out0.scalar_type() == at::kBFloat16, "bf16 epilogue output must be bf16");
  }
  if (epi == EPI_RELU_ROPE && e.freq) TORCH_CHECK(e.out1, "RoPE epilogue needs out1");
  if (epi == EPI_GATE) TORCH_CHECK(e.aux0, "gate epilogue needs aux0 (x)");
  if (epi == EPI_DEC_BWD) TORCH_CHECK(e.aux0 && e.aux1 && e.out1, "decoder backward epilogue needs x, yn, out1");
  if (epi == EPI_DQ) TORCH_CHECK(e.aux0, "dq epilogue needs dx_part (carrying the x mask)");
  if (epi == EPI_RELU_ROPE || epi == EPI_GATE || epi == EPI_DEC_BWD || epi == EPI_DQ) {
    TORCH_CHECK(bn == 128 || bn == 256, "TMA-epilogue modes use tile N = 128 or 256");
    TORCH_CHECK(!causal_skip, "TMA-epilogue modes have no zero tiles");
    // columns per epilogue chunk: 32 for the 16-warp x-projection epilogue, else 64
    const uint32_t cw = (epi == EPI_RELU_ROPE || bn == 256) ? 32 : 64;
    p.to0 = encode_out_map(e.out0, N, M, ld, Z1, sz1, Z2, sz2, cw);
    if (e.out1) p.to1 = encode_out_map(e.out1, N, M, ld, Z1, sz1, Z2, sz2, cw);
    if (e.aux0) p.tx0 = encode_out_map(e.aux0, N, M, ld, Z1, sz1, Z2, sz2, cw);
    if (e.rope_tma) p.tx0 = encode_table_map(rope_tab->data_ptr(), Nh / 2, T, cw);
    if (e.aux1) p.tx1 = encode_out_map(e.aux1, N, M, ld, Z1, sz1, Z2, sz2, cw);
  }
  hit->fn(p, at::cuda::getCurrentCUDAStream(dev).stream(), dev);
}

namespace {
// (cos, sin) of the RoPE phase 2*pi*frac(pos * freq[2j]) as half2, pos = pos0 + t.
__global__ void rope_table_kernel(const float* __restrict__ freq, int pos0, int T, int half_nh,
                                  uint32_t* __restrict__ out) {
  const long long n = (long long)T * half_nh;
  for (long long k = (long long)blockIdx.x * blockDim.x + threadIdx.x; k < n; k += (long long)gridDim.x * blockDim.x) {
    const int t = (int)(k / half_nh), j = (int)(k % half_nh);
    float c, s;
    rope_cs((float)(pos0 + t), freq[2 * j], c, s);
    const __half2 h = __floats2half2_rn(c, s);
    out[k] = *reinterpret_cast<const uint32_t*>(&h);
  }
}
}  // namespace

// Fill the half2 RoPE table [T, Nh/2] read by the x-projection and dQ epilogues.
void rope_table(const at::Tensor& freq, int64_t pos0, int64_t T, const at::Tensor& out) {
  TORCH_CHECK(freq.scalar_type() == at::kFloat && out.scalar_type() == at::kInt, "fp32 freq, int32 table");
  const int64_t half_nh = freq.numel() / 2;
  TORCH_CHECK(out.numel() >= T * half_nh, "rope table too small");
  c10::cuda::CUDAGuard guard(freq.get_device());
  rope_table_kernel<<<148 * 4, 256, 0, at::cuda::getCurrentCUDAStream(freq.get_device()).stream()>>>(
      freq.data_ptr<float>(), (int)pos0, (int)T, (int)half_nh, reinterpret_cast<uint32_t*>(out.data_ptr()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace bd
