// comm.cu — data-parallel gradient communication over NVLink peer memory.
//
// Every rank allocates one symmetric region (same layout on every GPU) with cudaMalloc
// and shares it through CUDA IPC; each rank then holds device pointers to all peers'
// regions. The gradient step of data-parallel training becomes three launches:
//
//   1. barrier(0)        every rank's gradients are final (system-scope release/acquire)
//   2. reduce_adamw      rank r owns elements [lo_r, hi_r): it sums that slice of every
//                        peer's gradient with plain P2P loads (a reduce-scatter), applies
//                        AdamW to its fp32 master slice and local moments, and stores the
//                        updated fp32 master and bf16 GEMM shadow into EVERY peer's region
//                        (an all-gather by P2P stores) — one pass, no staging copies
//   3. barrier(1)        every peer's slice has landed before the next forward starts
//
// This replaces the reference's one all-reduce per parameter tensor after the backward
// (burn_dragon_language/src/train/schedule.rs:10348-10457) followed by a full optimizer
// step on every rank. Loads are ordinary loads: no TMA, no multicast. Every wait on a
// peer flag is bounded by a %globaltimer deadline and reports through an error word.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_bf16.h>
#include <torch/extension.h>

#include <algorithm>
#include <vector>

namespace bd {
namespace {

constexpr int kMaxRanks = 8;
constexpr unsigned long long kPeerWaitNs = 5000000000ull;  // 5 s

struct PeerPtrs {
  float* grad[kMaxRanks];
  float* param[kMaxRanks];
  __nv_bfloat16* shadow[kMaxRanks];
  unsigned int* flags[kMaxRanks];
};

__device__ __forceinline__ unsigned long long gtimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ unsigned int ld_acquire_sys(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(unsigned int* p, unsigned int v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// flags layout on every rank: [phase][src rank] epoch counters, then this rank's own
// step counter at [2 * kMaxRanks]. The epoch comes from that device counter (phase 0
// advances it), so a captured CUDA graph replays with a fresh epoch every step.
__global__ void peer_barrier_kernel(PeerPtrs pp, int rank, int world, int phase, int* err) {
  const int t = threadIdx.x;
  __shared__ unsigned int s_epoch;
  unsigned int* ctr = pp.flags[rank] + 2 * kMaxRanks;
  if (t == 0) {
    unsigned int e = *ctr;
    if (phase == 0) {
      e += 1;
      *ctr = e;
    }
    s_epoch = e;
  }
  __threadfence_system();
  __syncthreads();
  const unsigned int epoch = s_epoch;
  if (t < world) st_release_sys(pp.flags[t] + phase * kMaxRanks + rank, epoch);
  if (t < world) {
    const unsigned int* mine = pp.flags[rank] + phase * kMaxRanks + t;
    const unsigned long long t0 = gtimer();
    while (ld_acquire_sys(mine) < epoch) {
      if (gtimer() - t0 > kPeerWaitNs) {
        atomicCAS(err, 0, 100 + phase);
        break;
      }
    }
  }
  __syncthreads();
}

__global__ void reduce_adamw_kernel(PeerPtrs pp, int rank, int world, long long lo, long long hi, float* m,
                                    float* v, float lr, float b1, float b2, float eps, float wd, float bc1, float bc2,
                                    const float* hyper, float inv_world) {
  if (hyper) {
    lr = hyper[0];
    bc1 = hyper[1];
    bc2 = hyper[2];
  }
  // 4 elements per thread step (lo, hi are multiples of 4)
  for (long long i = lo + 4ll * ((long long)blockIdx.x * blockDim.x + threadIdx.x); i < hi;
       i += 4ll * (long long)gridDim.x * blockDim.x) {
    float4 g = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int r = 0; r < kMaxRanks; ++r) {
      if (r >= world) break;
      const int src = (rank + r) % world;  // stagger the peers each rank starts with
      const float4 x = *reinterpret_cast<const float4*>(pp.grad[src] + i);
      g.x += x.x;
      g.y += x.y;
      g.z += x.z;
      g.w += x.w;
    }
    const long long s = i - lo;
    float4 p = *reinterpret_cast<const float4*>(pp.param[rank] + i);
    float4 mm = *reinterpret_cast<float4*>(m + s);
    float4 vv = *reinterpret_cast<float4*>(v + s);
    float gi[4] = {g.x * inv_world, g.y * inv_world, g.z * inv_world, g.w * inv_world};
    float* pe = &p.x;
    float* me = &mm.x;
    float* ve = &vv.x;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      me[k] = b1 * me[k] + (1.f - b1) * gi[k];
      ve[k] = b2 * ve[k] + (1.f - b2) * gi[k] * gi[k];
      pe[k] = pe[k] * (1.f - lr * wd) - lr * (me[k] / bc1) / (sqrtf(ve[k] / bc2) + eps);
    }
    *reinterpret_cast<float4*>(m + s) = mm;
    *reinterpret_cast<float4*>(v + s) = vv;
    __nv_bfloat162 h0 = __floats2bfloat162_rn(p.x, p.y), h1 = __floats2bfloat162_rn(p.z, p.w);
    uint2 hb;
    hb.x = *reinterpret_cast<unsigned int*>(&h0);
    hb.y = *reinterpret_cast<unsigned int*>(&h1);
#pragma unroll
    for (int r = 0; r < kMaxRanks; ++r) {
      if (r >= world) break;
      *reinterpret_cast<float4*>(pp.param[r] + i) = p;
      *reinterpret_cast<uint2*>(pp.shadow[r] + i) = hb;
    }
  }
}

// Plain all-reduce (mean) over the symmetric gradient region: rank r reduces its slice
// and writes the mean back into every peer's gradient region.
__global__ void reduce_mean_kernel(PeerPtrs pp, int rank, int world, long long lo, long long hi, float inv_world) {
  for (long long i = lo + 4ll * ((long long)blockIdx.x * blockDim.x + threadIdx.x); i < hi;
       i += 4ll * (long long)gridDim.x * blockDim.x) {
    float4 g = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int r = 0; r < world; ++r) {
      const float4 x = *reinterpret_cast<const float4*>(pp.grad[(rank + r) % world] + i);
      g.x += x.x;
      g.y += x.y;
      g.z += x.z;
      g.w += x.w;
    }
    g.x *= inv_world;
    g.y *= inv_world;
    g.z *= inv_world;
    g.w *= inv_world;
    for (int r = 0; r < world; ++r) *reinterpret_cast<float4*>(pp.grad[r] + i) = g;
  }
}

// Tensor-parallel sum, second half: every rank's GEMM epilogue stored its partial rows
// of owner o into o's slot buffer (slot s = source rank, [rows, D] each). The owner
// sums its W slots and stores the total into every rank's destination rows (an
// all-gather by P2P stores).
struct DstPtrs {
  float* dst[kMaxRanks];
};

__global__ void tp_reduce_gather_kernel(const float* __restrict__ slots, DstPtrs dp, int world, int rank,
                                        long long rows, long long valid_rows, int D, long long slot_stride) {
  const long long n4 = valid_rows * D / 4;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (long long)gridDim.x * blockDim.x) {
    const long long e = 4 * i;
    float4 acc = *reinterpret_cast<const float4*>(slots + e);
    for (int s = 1; s < world; ++s) {
      const float4 x = *reinterpret_cast<const float4*>(slots + s * slot_stride + e);
      acc.x += x.x;
      acc.y += x.y;
      acc.z += x.z;
      acc.w += x.w;
    }
    const long long o = rank * rows * D + e;
    for (int r = 0; r < world; ++r) {
      const int t = (rank + r) % world;  // stagger the destinations
      *reinterpret_cast<float4*>(dp.dst[t] + o) = acc;
    }
  }
}

// Row scatter for a tensor-parallel sum of an [M, D] partial that is already in local
// memory: row r goes to owner r / rows, into slot `rank` of that owner (P2P stores).
__global__ void tp_scatter_rows_kernel(const float* __restrict__ src, DstPtrs slots, int rank, long long rows,
                                       long long M, int D, long long slot_stride) {
  const long long n4 = M * D / 4;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (long long)gridDim.x * blockDim.x) {
    const long long e = 4 * i;
    const long long r = e / D;
    const int owner = (int)(r / rows);
    const float4 x = *reinterpret_cast<const float4*>(src + e);
    *reinterpret_cast<float4*>(slots.dst[owner] + rank * slot_stride + (r - owner * rows) * D + (e - r * D)) = x;
  }
}

PeerPtrs make_ptrs(const std::vector<int64_t>& grad, const std::vector<int64_t>& param,
                   const std::vector<int64_t>& shadow, const std::vector<int64_t>& flags) {
  PeerPtrs pp;
  memset(&pp, 0, sizeof(pp));
  const size_t w = grad.size();
  TORCH_CHECK(w >= 1 && w <= kMaxRanks && param.size() == w && shadow.size() == w && flags.size() == w,
              "peer pointer lists must have one entry per rank (<= 8)");
  for (size_t r = 0; r < w; ++r) {
    pp.grad[r] = reinterpret_cast<float*>(grad[r]);
    pp.param[r] = reinterpret_cast<float*>(param[r]);
    pp.shadow[r] = reinterpret_cast<__nv_bfloat16*>(shadow[r]);
    pp.flags[r] = reinterpret_cast<unsigned int*>(flags[r]);
  }
  return pp;
}

}  // namespace

// ---- symmetric memory: raw allocations (exact IPC base pointers)
int64_t sym_alloc(int64_t bytes, int64_t device) {
  c10::cuda::CUDAGuard g((c10::DeviceIndex)device);
  void* p = nullptr;
  C10_CUDA_CHECK(cudaMalloc(&p, (size_t)bytes));
  C10_CUDA_CHECK(cudaMemset(p, 0, (size_t)bytes));
  return reinterpret_cast<int64_t>(p);
}

void sym_free(int64_t ptr, int64_t device) {
  c10::cuda::CUDAGuard g((c10::DeviceIndex)device);
  C10_CUDA_CHECK(cudaFree(reinterpret_cast<void*>(ptr)));
}

std::vector<int64_t> ipc_handle(int64_t ptr, int64_t device) {
  c10::cuda::CUDAGuard g((c10::DeviceIndex)device);
  cudaIpcMemHandle_t h;
  C10_CUDA_CHECK(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(ptr)));
  std::vector<int64_t> out(sizeof(h));
  const unsigned char* b = reinterpret_cast<const unsigned char*>(&h);
  for (size_t i = 0; i < sizeof(h); ++i) out[i] = b[i];
  return out;
}

int64_t ipc_open(std::vector<int64_t> handle, int64_t device) {
  c10::cuda::CUDAGuard g((c10::DeviceIndex)device);
  cudaIpcMemHandle_t h;
  TORCH_CHECK(handle.size() == sizeof(h), "bad IPC handle size");
  unsigned char* b = reinterpret_cast<unsigned char*>(&h);
  for (size_t i = 0; i < sizeof(h); ++i) b[i] = (unsigned char)handle[i];
  void* p = nullptr;
  C10_CUDA_CHECK(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  return reinterpret_cast<int64_t>(p);
}

void ipc_close(int64_t ptr, int64_t device) {
  c10::cuda::CUDAGuard g((c10::DeviceIndex)device);
  C10_CUDA_CHECK(cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr)));
}

at::Tensor wrap_ptr(int64_t ptr, int64_t numel, int64_t dtype_code, int64_t device) {
  const at::ScalarType st = dtype_code == 0 ? at::kFloat : (dtype_code == 1 ? at::kBFloat16 : at::kInt);
  return torch::from_blob(reinterpret_cast<void*>(ptr), {numel},
                          at::TensorOptions().dtype(st).device(at::kCUDA, (c10::DeviceIndex)device));
}

void peer_barrier(std::vector<int64_t> grad, std::vector<int64_t> param, std::vector<int64_t> shadow,
                  std::vector<int64_t> flags, int64_t rank, int64_t phase, const at::Tensor& err) {
  PeerPtrs pp = make_ptrs(grad, param, shadow, flags);
  auto st = at::cuda::getCurrentCUDAStream(err.get_device()).stream();
  peer_barrier_kernel<<<1, 32, 0, st>>>(pp, (int)rank, (int)grad.size(), (int)phase, err.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void reduce_adamw(std::vector<int64_t> grad, std::vector<int64_t> param, std::vector<int64_t> shadow,
                  std::vector<int64_t> flags, int64_t rank, int64_t lo, int64_t hi, const at::Tensor& m,
                  const at::Tensor& v, double lr, double b1, double b2, double eps, double wd, double bc1, double bc2,
                  const c10::optional<at::Tensor>& hyper) {
  PeerPtrs pp = make_ptrs(grad, param, shadow, flags);
  TORCH_CHECK(lo % 4 == 0 && hi % 4 == 0, "shard bounds must be multiples of 4");
  TORCH_CHECK(m.numel() >= hi - lo && v.numel() >= hi - lo, "moment shards too small");
  auto st = at::cuda::getCurrentCUDAStream(m.get_device()).stream();
  const int world = (int)grad.size();
  reduce_adamw_kernel<<<148 * 4, 256, 0, st>>>(pp, (int)rank, world, lo, hi, m.data_ptr<float>(), v.data_ptr<float>(),
                                               (float)lr, (float)b1, (float)b2, (float)eps, (float)wd, (float)bc1,
                                               (float)bc2, hyper ? hyper->data_ptr<float>() : nullptr,
                                               1.0f / (float)world);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void tp_reduce_gather(const at::Tensor& slots, std::vector<int64_t> dst, int64_t rank, int64_t rows, int64_t M,
                      int64_t D, int64_t slot_stride) {
  const int world = (int)dst.size();
  TORCH_CHECK(world >= 1 && world <= kMaxRanks, "1..8 ranks");
  TORCH_CHECK(slots.scalar_type() == at::kFloat && slots.is_contiguous() && D % 4 == 0, "fp32 slots, D % 4 == 0");
  DstPtrs dp;
  memset(&dp, 0, sizeof(dp));
  for (int r = 0; r < world; ++r) dp.dst[r] = reinterpret_cast<float*>(dst[r]);
  const long long valid = std::max<long long>(0, std::min<long long>(rows, M - rank * rows));
  auto st = at::cuda::getCurrentCUDAStream(slots.get_device()).stream();
  tp_reduce_gather_kernel<<<148 * 2, 256, 0, st>>>(slots.data_ptr<float>(), dp, world, (int)rank, rows, valid,
                                                   (int)D, slot_stride);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void tp_scatter_rows(const at::Tensor& src, std::vector<int64_t> slots, int64_t rank, int64_t rows, int64_t M,
                     int64_t D, int64_t slot_stride) {
  const int world = (int)slots.size();
  TORCH_CHECK(world >= 1 && world <= kMaxRanks && rows * world >= M, "1..8 ranks covering the rows");
  TORCH_CHECK(src.scalar_type() == at::kFloat && src.is_contiguous() && src.numel() >= M * D && D % 4 == 0,
              "fp32 contiguous [M, D] source, D % 4 == 0");
  DstPtrs dp;
  memset(&dp, 0, sizeof(dp));
  for (int r = 0; r < world; ++r) dp.dst[r] = reinterpret_cast<float*>(slots[r]);
  auto st = at::cuda::getCurrentCUDAStream(src.get_device()).stream();
  tp_scatter_rows_kernel<<<148 * 2, 256, 0, st>>>(src.data_ptr<float>(), dp, (int)rank, rows, M, (int)D,
                                                  slot_stride);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void reduce_mean(std::vector<int64_t> grad, std::vector<int64_t> flags, int64_t rank, int64_t lo, int64_t hi,
                 const at::Tensor& err) {
  std::vector<int64_t> z(grad.size(), 0);
  PeerPtrs pp = make_ptrs(grad, z, z, flags);
  auto st = at::cuda::getCurrentCUDAStream(err.get_device()).stream();
  reduce_mean_kernel<<<148 * 4, 256, 0, st>>>(pp, (int)rank, (int)grad.size(), lo, hi, 1.0f / (float)grad.size());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace bd
