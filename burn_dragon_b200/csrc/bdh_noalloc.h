// bdh_noalloc.h — C interface of the allocation-free decoder-merge entry point.
//
// This interface has no counterpart in the reference; it is an addition of this library.
//
// bdh_decoder_merge_noalloc computes v_out = LN(v + LN(yn @ dec)) for callers that must
// not allocate device memory (a runtime that plans every buffer before it starts and
// forbids allocation while it runs, a plugin inside a framework that owns the CUDA
// allocator, plain C reaching this library through an FFI). Its split-K scratch is a
// 32 MiB device array built into the library; the caller passes inputs and outputs.
// The full contract is in the comment at the top of noalloc_decoder.cu.
#ifndef BDH_NOALLOC_H_
#define BDH_NOALLOC_H_

#include <stddef.h>
#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

// Return codes of bdh_decoder_merge_noalloc.
enum {
  BDH_NOALLOC_OK = 0,
  BDH_NOALLOC_ERR_ARGS = 1,            // null pointer, unsupported D, N % 64 or D % 32, stream of another device
  BDH_NOALLOC_ERR_TOO_LARGE = 2,       // splits * M * D * 4 bytes exceed the built-in scratch
  BDH_NOALLOC_ERR_SETUP = 3,           // the scratch array's device address could not be resolved
  BDH_NOALLOC_ERR_CUDA = 4,            // a CUDA call or kernel launch of this call failed
  BDH_NOALLOC_ERR_KERNEL_TIMEOUT = 5,  // the GEMM reported a bounded-wait timeout (check != 0 only)
};

// v_out = LN(v + LN(yn @ dec)), one LayerNorm (gamma, beta, eps) used twice.
//   yn [M, N] bf16 row-major, dec [N, D] bf16 row-major, v / v_out [M, D] fp32,
//   gamma / beta [D] fp32, v_out_bf16 [M, D] bf16 or NULL. D in {32, 64, 128, 256},
//   N % 64 == 0, 1 <= splits <= N / 64 (rounded down to the count that covers N).
// Enqueued on `stream`, which must belong to the current device. With check != 0 the
// call synchronizes the stream and reports a kernel timeout; with check == 0 it returns
// after enqueueing and the caller reads the device word bdh_noalloc_error_word() later
// (non-zero: that call's result is invalid; the next call clears it).
int bdh_decoder_merge_noalloc(const void* yn, const void* dec, const float* v, const float* gamma,
                              const float* beta, float* v_out, void* v_out_bf16, int M, int N, int D, int splits,
                              float eps, int check, cudaStream_t stream);

// Text for a return code.
const char* bdh_noalloc_error_string(int code);

// Size of the built-in scratch array in bytes (the limit on splits * M * D * 4).
size_t bdh_noalloc_scratch_bytes(void);

// Device address of the current device's kernel error word (an int), resolved like the
// scratch array; NULL if that fails. Valid for the life of the process.
int* bdh_noalloc_error_word(void);

#ifdef __cplusplus
}
#endif

#endif  // BDH_NOALLOC_H_
