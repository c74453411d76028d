// noalloc_decoder.cu — an allocation-free C entry point for the BDH decoder product
// followed by the residual merge:  v' = LN(v + LN(yn @ E)).
//
// This entry point has no counterpart in the reference; it is an addition of this
// library.
//
// Who it is for: code that drives the GPU but must not allocate device memory itself —
// for example a host runtime that pre-plans every buffer up front and forbids
// allocation once it runs (a real-time / serving loop with a fixed memory budget), a
// plugin loaded into another framework that owns the CUDA allocator, or a caller
// reaching this library from C through a foreign-function interface without any
// PyTorch allocator at hand. The regular path (ops.gemm + rowwise.cu tail_fwd) needs a
// split-K partial buffer that the caller allocates through torch; this variant keeps
// that scratch in a fixed device array compiled into the library instead.
//
// Contract:
//  * The caller passes all inputs and outputs as device pointers. The function calls
//    no cudaMalloc, cudaFree or any allocating library routine.
//  * Scratch is the file-scope device array `g_noalloc_scratch`, 32 MiB on every GPU
//    that loads the library, held until the process exits. Requests whose split-K
//    partials (splits * M * D fp32 values) do not fit are rejected with
//    BDH_NOALLOC_ERR_TOO_LARGE before anything is launched.
//  * The first call on a device looks the scratch array up with cudaGetSymbolAddress
//    (once per device, with that device current). Make that first call before any
//    stream capture begins.
//  * All calls share the one scratch array, which keeps the previous call's contents.
//    Every partial element is rewritten on each call, so nothing in it has to start at
//    zero; the device error word is cleared at the start of each call. Calls that
//    overlap on the GPU (different streams, or different host threads on one device)
//    race on the scratch array and must be serialized by the caller.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cstring>
#include <exception>

#include "bdh_noalloc.h"
#include "gemm_sm100.cuh"
#include "gemm_table.h"

namespace {

constexpr size_t kScratchBytes = 32u << 20;  // 32 MiB
static __device__ __align__(256) float g_noalloc_scratch[kScratchBytes / sizeof(float)];
static __device__ int g_noalloc_err;

constexpr int kMaxDevices = 64;
float* g_scratch_ptr[kMaxDevices] = {nullptr};
int* g_err_ptr[kMaxDevices] = {nullptr};

// Per-device set-up: resolve the device addresses of the scratch array and error word.
// Two host threads making their first call on one device at once both resolve the same
// addresses and store the same values, so the unsynchronized cache is benign.
int setup_device(int dev) {
  if (g_scratch_ptr[dev] != nullptr) return BDH_NOALLOC_OK;
  void* s = nullptr;
  void* e = nullptr;
  if (cudaGetSymbolAddress(&s, g_noalloc_scratch) != cudaSuccess || s == nullptr) return BDH_NOALLOC_ERR_SETUP;
  if (cudaGetSymbolAddress(&e, g_noalloc_err) != cudaSuccess || e == nullptr) return BDH_NOALLOC_ERR_SETUP;
  g_err_ptr[dev] = static_cast<int*>(e);
  g_scratch_ptr[dev] = static_cast<float*>(s);
  return BDH_NOALLOC_OK;
}

bool encode(CUtensorMap* m, const void* base, uint64_t inner, uint64_t outer, uint64_t stride_elems,
            uint32_t box_inner, uint32_t box_outer) {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (fn == nullptr) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || ptr == nullptr)
      return false;
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  const uint64_t plane = outer * stride_elems * 2;
  cuuint64_t dims[4] = {inner, outer, 1, 1};
  cuuint64_t strides[3] = {stride_elems * 2, plane, plane};
  cuuint32_t box[4] = {box_inner, box_outer, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

__device__ __forceinline__ float wsum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// One warp per row: m = sum of the split partials in scratch, v' = LN(v + LN(m)).
template <int VPL>
__global__ void merge_rows_kernel(const float* __restrict__ partial, int splits, long long split_stride,
                                  const float* __restrict__ v, long long rows, int D, const float* __restrict__ gamma,
                                  const float* __restrict__ beta, float eps, float* __restrict__ out32,
                                  __nv_bfloat16* __restrict__ out16) {
  const int lane = threadIdx.x % 32;
  const long long row = (long long)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  if (row >= rows) return;
  float m[VPL];
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    float acc = 0.f;
    for (int k = 0; k < splits; ++k) acc += partial[k * split_stride + row * D + lane + 32 * i];
    m[i] = acc;
    s += acc;
  }
  float mean = wsum(s) / D, q = 0.f;
#pragma unroll
  for (int i = 0; i < VPL; ++i) q += (m[i] - mean) * (m[i] - mean);
  float rstd = rsqrtf(wsum(q) / D + eps);
  s = 0.f;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int c = lane + 32 * i;
    m[i] = v[row * D + c] + (m[i] - mean) * rstd * gamma[c] + beta[c];
    s += m[i];
  }
  mean = wsum(s) / D;
  q = 0.f;
#pragma unroll
  for (int i = 0; i < VPL; ++i) q += (m[i] - mean) * (m[i] - mean);
  rstd = rsqrtf(wsum(q) / D + eps);
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int c = lane + 32 * i;
    const float y = (m[i] - mean) * rstd * gamma[c] + beta[c];
    out32[row * D + c] = y;
    if (out16) out16[row * D + c] = __float2bfloat16_rn(y);
  }
}

}  // namespace

extern "C" {

// Human-readable text for a return code of bdh_decoder_merge_noalloc.
const char* bdh_noalloc_error_string(int code) {
  switch (code) {
    case BDH_NOALLOC_OK: return "ok";
    case BDH_NOALLOC_ERR_ARGS: return "invalid arguments (null pointer, unsupported D, or N/D not multiples of 64/32)";
    case BDH_NOALLOC_ERR_TOO_LARGE: return "splits*M*D*4 bytes exceeds the 32 MiB built-in scratch";
    case BDH_NOALLOC_ERR_SETUP: return "cudaGetSymbolAddress of the built-in scratch failed";
    case BDH_NOALLOC_ERR_CUDA: return "a CUDA call or kernel launch failed";
    case BDH_NOALLOC_ERR_KERNEL_TIMEOUT: return "the GEMM kernel reported a bounded-wait timeout";
    default: return "unknown error";
  }
}

// Bytes of built-in scratch available to bdh_decoder_merge_noalloc.
size_t bdh_noalloc_scratch_bytes(void) { return kScratchBytes; }

// Device address of the current device's error word, for callers that pass check == 0.
int* bdh_noalloc_error_word(void) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  if (setup_device(dev) != BDH_NOALLOC_OK) return nullptr;
  return g_err_ptr[dev];
}

// v_out = LN(v + LN(yn @ dec)) with one shared LayerNorm (gamma, beta, eps).
//   yn    [M, N]  bf16, row-major      dec   [N, D] bf16, row-major
//   v     [M, D]  fp32                 gamma, beta [D] fp32
//   v_out [M, D]  fp32                 v_out_bf16 [M, D] bf16 or NULL
// `splits` divides the K = N reduction across CTAs (1..N/64); the partial products live
// in the built-in scratch. Enqueued on `stream` (a stream of the current device); returns
// 0 or a code of bdh_noalloc_error_string. The device error word is read back only when
// `check` != 0 (that read synchronizes the stream); with check == 0 a GEMM timeout is
// not reported here, and the caller reads bdh_noalloc_error_word() later instead.
int bdh_decoder_merge_noalloc(const void* yn, const void* dec, const float* v, const float* gamma,
                              const float* beta, float* v_out, void* v_out_bf16, int M, int N, int D, int splits,
                              float eps, int check, cudaStream_t stream) {
  if (!yn || !dec || !v || !gamma || !beta || !v_out || M <= 0 || N <= 0 || D <= 0 || splits <= 0)
    return BDH_NOALLOC_ERR_ARGS;
  if (N % 64 || D % 32 || (D / 32 != 1 && D / 32 != 2 && D / 32 != 4 && D / 32 != 8)) return BDH_NOALLOC_ERR_ARGS;
  const int KB = N / 64;
  if (splits > KB) return BDH_NOALLOC_ERR_ARGS;
  const int per = (KB + splits - 1) / splits;
  const int real_splits = (KB + per - 1) / per;
  if ((size_t)real_splits * (size_t)M * (size_t)D * sizeof(float) > kScratchBytes) return BDH_NOALLOC_ERR_TOO_LARGE;
  // an error left by the caller's earlier work is not this call's: drain it first
  (void)cudaGetLastError();
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return BDH_NOALLOC_ERR_CUDA;
#if CUDART_VERSION >= 12080
  if (stream != nullptr) {
    int sdev = -1;
    if (cudaStreamGetDevice(stream, &sdev) != cudaSuccess) return BDH_NOALLOC_ERR_CUDA;
    if (sdev != dev) return BDH_NOALLOC_ERR_ARGS;
  }
#endif
  int rc = setup_device(dev);
  if (rc != BDH_NOALLOC_OK) return rc;
  float* scratch = g_scratch_ptr[dev];
  int* err = g_err_ptr[dev];
  if (cudaMemsetAsync(err, 0, sizeof(int), stream) != cudaSuccess) return BDH_NOALLOC_ERR_CUDA;

  const int bn = (D % 256 == 0) ? 256 : (D % 128 == 0 ? 128 : 64);
  const bd::Entry* hit = nullptr;
  for (int i = 0; i < bd::kGemmTableBSize; ++i) {
    const bd::Entry& en = bd::kGemmTableB[i];
    if (en.bn == bn && !en.a_mn && en.b_mn && en.epi == bd::EPI_F32) hit = &en;
  }
  if (hit == nullptr) return BDH_NOALLOC_ERR_ARGS;

  bd::GemmParams p;
  std::memset(&p, 0, sizeof(p));
  if (!encode(&p.ta, yn, (uint64_t)N, (uint64_t)M, (uint64_t)N, 64, 128)) return BDH_NOALLOC_ERR_CUDA;
  if (!encode(&p.tb, dec, (uint64_t)D, (uint64_t)N, (uint64_t)D, 64, 64)) return BDH_NOALLOC_ERR_CUDA;
  p.M = M;
  p.N = D;
  p.K = N;
  p.Z1 = 1;
  p.Z2 = 1;
  p.tiles_m = (M + 127) / 128;
  p.tiles_n = (D + bn - 1) / bn;
  p.kb_per_split = per;
  p.splits = real_splits;
  p.err = err;
  p.e.out0 = scratch;
  p.e.ld = D;
  p.e.split_stride = (long long)M * D;
  p.e.alpha = 1.0f;
  p.e.T = 1;
  p.e.Nh = 1;
  try {
    hit->fn(p, stream, dev);
  } catch (const std::exception&) {
    return BDH_NOALLOC_ERR_CUDA;
  }
  const int warps = 8;
  const int blocks = (M + warps - 1) / warps;
  auto* o16 = static_cast<__nv_bfloat16*>(v_out_bf16);
  switch (D / 32) {
    case 1: merge_rows_kernel<1><<<blocks, warps * 32, 0, stream>>>(scratch, real_splits, p.e.split_stride, v, M, D, gamma, beta, eps, v_out, o16); break;
    case 2: merge_rows_kernel<2><<<blocks, warps * 32, 0, stream>>>(scratch, real_splits, p.e.split_stride, v, M, D, gamma, beta, eps, v_out, o16); break;
    case 4: merge_rows_kernel<4><<<blocks, warps * 32, 0, stream>>>(scratch, real_splits, p.e.split_stride, v, M, D, gamma, beta, eps, v_out, o16); break;
    default: merge_rows_kernel<8><<<blocks, warps * 32, 0, stream>>>(scratch, real_splits, p.e.split_stride, v, M, D, gamma, beta, eps, v_out, o16); break;
  }
  if (cudaGetLastError() != cudaSuccess) return BDH_NOALLOC_ERR_CUDA;
  if (check) {
    int host_err = 0;
    if (cudaMemcpyAsync(&host_err, err, sizeof(int), cudaMemcpyDeviceToHost, stream) != cudaSuccess ||
        cudaStreamSynchronize(stream) != cudaSuccess)
      return BDH_NOALLOC_ERR_CUDA;
    if (host_err != 0) return BDH_NOALLOC_ERR_KERNEL_TIMEOUT;
  }
  return BDH_NOALLOC_OK;
}

}  // extern "C"
