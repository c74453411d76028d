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
#include <type_traits>
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


// ---------------------------------------------------------------------------------------
// The data-parallel optimizer step over NVLink, bf16 transport (ddp_step):
//
//   every rank   casts its fp32 gradients into its symmetric bf16 gradient buffer
//   barrier(0)
//   rank r       owns elements [lo_r, hi_r): sums that slice of every peer's bf16 gradient
//                (fp32 accumulation, peers loaded together so their latencies overlap),
//                applies AdamW to its fp32 master slice (kept only here) and its moment
//                shard, and stores the new bf16 weights into every peer's shadow buffer
//   barrier(1)
//
// Bytes over NVLink per rank: (W-1)/W * P * 2 in and the same out (P = parameters), a
// third of the fp32-gradient, fp32-master step. With global-norm clipping the sum runs
// first into a local fp32 shard (ddp_reduce), the ranks exchange their shard's sum of
// squares (ddp_norm_exchange), and the update reads the clipped local shard (ddp_apply).
struct DdpPtrs {
  const void* grad[kMaxRanks];  // bf16 (or fp32) gradient buffer of every rank
  __nv_bfloat16* shadow[kMaxRanks];
  float* master[kMaxRanks];     // fp32 master of every rank, or null: not gathered
};

template <typename GT>
struct Vec8 {
  static __device__ __forceinline__ void load(const GT* p, float (&o)[8]);
};
template <>
struct Vec8<__nv_bfloat16> {
  static __device__ __forceinline__ void load(const __nv_bfloat16* p, float (&o)[8]) {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __bfloat1622float2(h[i]);
      o[2 * i] = f.x;
      o[2 * i + 1] = f.y;
    }
  }
};
template <>
struct Vec8<float> {
  static __device__ __forceinline__ void load(const float* p, float (&o)[8]) {
    const float4 a = *reinterpret_cast<const float4*>(p);
    const float4 b = *reinterpret_cast<const float4*>(p + 4);
    o[0] = a.x; o[1] = a.y; o[2] = a.z; o[3] = a.w;
    o[4] = b.x; o[5] = b.y; o[6] = b.z; o[7] = b.w;
  }
};

// Sum of the W ranks' gradients for 8 elements at i, every peer's load issued before any
// is used (the loop bound is a template constant, so the loads are not serialized behind
// the adds of earlier peers).
template <int W, typename GT>
__device__ __forceinline__ void peer_sum8(const DdpPtrs& pp, int rank, long long i, float (&g)[8]) {
  float x[W][8];
#pragma unroll
  for (int r = 0; r < W; ++r) {
    int src = rank + r;
    if (src >= W) src -= W;  // stagger the peer each rank starts with
    Vec8<GT>::load(reinterpret_cast<const GT*>(pp.grad[src]) + i, x[r]);
  }
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    float a = 0.f;
#pragma unroll
    for (int r = 0; r < W; ++r) a += x[r][k];
    g[k] = a;
  }
}

__device__ __forceinline__ float block_sum(float v) {
  __shared__ float red[32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x / 32, l = threadIdx.x % 32;
  if (l == 0) red[w] = v;
  __syncthreads();
  float t = 0.f;
  if (w == 0) {
    t = l < (int)(blockDim.x / 32) ? red[l] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
  }
  return t;  // valid in thread 0
}

// AdamW on 8 elements of the owned slice (hyper = {lr, 1 - b1^t, 1 - b2^t}): the fp32
// master at flat index i, the moments at shard index s; then the new weights as bf16
// into every rank's shadow at i.
__device__ __forceinline__ void adamw8_local(long long i, long long s, const float (&g)[8], float* __restrict__ master,
                                             float* __restrict__ m, float* __restrict__ v, float lr, float b1,
                                             float b2, float eps, float wd, float bc1, float bc2, float (&pv)[8]) {
  float mv[8], vv[8];
  Vec8<float>::load(master + i, pv);
  Vec8<float>::load(m + s, mv);
  Vec8<float>::load(v + s, vv);
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    mv[k] = b1 * mv[k] + (1.f - b1) * g[k];
    vv[k] = b2 * vv[k] + (1.f - b2) * g[k] * g[k];
    pv[k] = pv[k] * (1.f - lr * wd) - lr * (mv[k] / bc1) / (sqrtf(vv[k] / bc2) + eps);
  }
  *reinterpret_cast<float4*>(master + i) = make_float4(pv[0], pv[1], pv[2], pv[3]);
  *reinterpret_cast<float4*>(master + i + 4) = make_float4(pv[4], pv[5], pv[6], pv[7]);
  *reinterpret_cast<float4*>(m + s) = make_float4(mv[0], mv[1], mv[2], mv[3]);
  *reinterpret_cast<float4*>(m + s + 4) = make_float4(mv[4], mv[5], mv[6], mv[7]);
  *reinterpret_cast<float4*>(v + s) = make_float4(vv[0], vv[1], vv[2], vv[3]);
  *reinterpret_cast<float4*>(v + s + 4) = make_float4(vv[4], vv[5], vv[6], vv[7]);
}

__device__ __forceinline__ uint4 pack_bf16x8(const float (&pv)[8]) {
  uint4 hb;
  __nv_bfloat162 h;
  h = __floats2bfloat162_rn(pv[0], pv[1]); hb.x = *reinterpret_cast<unsigned int*>(&h);
  h = __floats2bfloat162_rn(pv[2], pv[3]); hb.y = *reinterpret_cast<unsigned int*>(&h);
  h = __floats2bfloat162_rn(pv[4], pv[5]); hb.z = *reinterpret_cast<unsigned int*>(&h);
  h = __floats2bfloat162_rn(pv[6], pv[7]); hb.w = *reinterpret_cast<unsigned int*>(&h);
  return hb;
}

template <int W>
__device__ __forceinline__ void adamw8_gather(const DdpPtrs& pp, int rank, long long i, long long s, float (&g)[8],
                                              float* __restrict__ master, float* __restrict__ m,
                                              float* __restrict__ v, float lr, float b1, float b2, float eps,
                                              float wd, float bc1, float bc2) {
  float pv[8];
  adamw8_local(i, s, g, master, m, v, lr, b1, b2, eps, wd, bc1, bc2, pv);
  const uint4 hb = pack_bf16x8(pv);
#pragma unroll
  for (int r = 0; r < W; ++r) {
    int dst = rank + r;
    if (dst >= W) dst -= W;
    *reinterpret_cast<uint4*>(pp.shadow[dst] + i) = hb;
    // buckets whose fp32 master the forward reads (embedding, norms, adapters): the new
    // master goes to every peer too (pp.master[rank] is this rank's own buffer)
    if (pp.master[0] != nullptr && dst != rank) {
      *reinterpret_cast<float4*>(pp.master[dst] + i) = make_float4(pv[0], pv[1], pv[2], pv[3]);
      *reinterpret_cast<float4*>(pp.master[dst] + i + 4) = make_float4(pv[4], pv[5], pv[6], pv[7]);
    }
  }
}

// Fused (no clipping): peer sum + AdamW + shadow all-gather in one pass. `master` is
// this rank's full fp32 buffer (the slice [lo, hi) is updated); m / v are shard-local.
template <int W, typename GT>
__global__ void __launch_bounds__(256) ddp_step_kernel(DdpPtrs pp, int rank, long long lo, long long hi,
                                                       float* __restrict__ master, float* __restrict__ m,
                                                       float* __restrict__ v, float b1, float b2, float eps,
                                                       float wd, const float* __restrict__ hyper,
                                                       const float* __restrict__ coef) {
  const float lr = hyper[0], bc1 = hyper[1], bc2 = hyper[2];
  const float scale = (1.0f / W) * (coef ? coef[0] : 1.0f);
  for (long long i = lo + 8ll * ((long long)blockIdx.x * blockDim.x + threadIdx.x); i < hi;
       i += 8ll * (long long)gridDim.x * blockDim.x) {
    float g[8];
    peer_sum8<W, GT>(pp, rank, i, g);
#pragma unroll
    for (int k = 0; k < 8; ++k) g[k] *= scale;
    adamw8_gather<W>(pp, rank, i, i - lo, g, master, m, v, lr, b1, b2, eps, wd, bc1, bc2);
  }
}

// Clipping, pass 1: the owned slice's mean gradient into a local fp32 shard, and its
// sum of squares into sumsq[0] (zeroed by the caller's stream before this launch).
template <int W, typename GT>
__global__ void __launch_bounds__(256) ddp_reduce_kernel(DdpPtrs pp, int rank, long long lo, long long hi,
                                                         float* __restrict__ gred, float* __restrict__ sumsq) {
  float acc = 0.f;
  for (long long i = lo + 8ll * ((long long)blockIdx.x * blockDim.x + threadIdx.x); i < hi;
       i += 8ll * (long long)gridDim.x * blockDim.x) {
    float g[8];
    peer_sum8<W, GT>(pp, rank, i, g);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      g[k] *= 1.0f / W;
      acc += g[k] * g[k];
    }
    float* o = gred + (i - lo);
    *reinterpret_cast<float4*>(o) = make_float4(g[0], g[1], g[2], g[3]);
    *reinterpret_cast<float4*>(o + 4) = make_float4(g[4], g[5], g[6], g[7]);
  }
  const float t = block_sum(acc);
  if (threadIdx.x == 0) atomicAdd(sumsq, t);
}

// Clipping, pass 2: AdamW from the local reduced shard, scaled by coef[0].
template <int W>
__global__ void __launch_bounds__(256) ddp_apply_kernel(DdpPtrs pp, int rank, long long lo, long long hi,
                                                        const float* __restrict__ gred, float* __restrict__ master,
                                                        float* __restrict__ m, float* __restrict__ v, float b1,
                                                        float b2, float eps, float wd,
                                                        const float* __restrict__ hyper,
                                                        const float* __restrict__ coef) {
  const float lr = hyper[0], bc1 = hyper[1], bc2 = hyper[2];
  const float c = coef[0];
  for (long long i = lo + 8ll * ((long long)blockIdx.x * blockDim.x + threadIdx.x); i < hi;
       i += 8ll * (long long)gridDim.x * blockDim.x) {
    float g[8];
    Vec8<float>::load(gred + (i - lo), g);
#pragma unroll
    for (int k = 0; k < 8; ++k) g[k] *= c;
    adamw8_gather<W>(pp, rank, i, i - lo, g, master, m, v, lr, b1, b2, eps, wd, bc1, bc2);
  }
}

// ---------------------------------------------------------------------------------------
// The same step through NVLink SHARP (NVLS) multicast addresses. The gradient, shadow and
// (gathered) master buffers are bound to one multicast object per buffer across the ranks;
// `multimem.ld_reduce` on a multicast address returns the sum of every rank's copy of those
// words, reduced inside the NVSwitch (one read per element crosses this GPU's links instead
// of W - 1), and `multimem.st` writes one copy that the switch delivers to every rank.
// bf16 gradients are summed with fp32 accumulation in the switch (.acc::f32) and arrive
// rounded to bf16 once; fp32 gradients are summed in fp32.
__device__ __forceinline__ void mc_sum8(const __nv_bfloat16* mc, float (&g)[8]) {
  uint32_t r[4];
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "l"(mc)
               : "memory");
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    g[2 * i] = __uint_as_float(r[i] << 16);
    g[2 * i + 1] = __uint_as_float(r[i] & 0xffff0000u);
  }
}

__device__ __forceinline__ void mc_sum8(const float* mc, float (&g)[8]) {
#pragma unroll
  for (int h = 0; h < 2; ++h)
    asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(g[4 * h]), "=f"(g[4 * h + 1]), "=f"(g[4 * h + 2]), "=f"(g[4 * h + 3])
                 : "l"(mc + 4 * h)
                 : "memory");
}

__device__ __forceinline__ void mc_store16(void* mc, uint4 v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(mc), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}

// AdamW on 8 elements from the summed gradient g; the new bf16 weights (and, for a gathered
// master, the fp32 values) leave through multicast stores.
__device__ __forceinline__ void adamw8_multicast(long long i, long long s, const float (&g)[8],
                                                 __nv_bfloat16* mc_shadow, float* mc_master,
                                                 float* __restrict__ master, float* __restrict__ m,
                                                 float* __restrict__ v, float lr, float b1, float b2, float eps,
                                                 float wd, float bc1, float bc2) {
  float pv[8];
  adamw8_local(i, s, g, master, m, v, lr, b1, b2, eps, wd, bc1, bc2, pv);
  mc_store16(mc_shadow + i, pack_bf16x8(pv));
  if (mc_master != nullptr) {
    mc_store16(mc_master + i, make_uint4(__float_as_uint(pv[0]), __float_as_uint(pv[1]), __float_as_uint(pv[2]),
                                         __float_as_uint(pv[3])));
    mc_store16(mc_master + i + 4, make_uint4(__float_as_uint(pv[4]), __float_as_uint(pv[5]), __float_as_uint(pv[6]),
                                             __float_as_uint(pv[7])));
  }
}

constexpr int kNvlsUnroll = 4;

template <typename GT>
__global__ void __launch_bounds__(256) ddp_step_nvls_kernel(const GT* mc_grad, __nv_bfloat16* mc_shadow,
                                                            float* mc_master, float inv_world, long long lo,
                                                            long long hi, float* __restrict__ master,
                                                            float* __restrict__ m, float* __restrict__ v, float b1,
                                                            float b2, float eps, float wd,
                                                            const float* __restrict__ hyper,
                                                            const float* __restrict__ coef) {
  const float lr = hyper[0], bc1 = hyper[1], bc2 = hyper[2];
  const float scale = inv_world * (coef ? coef[0] : 1.0f);
  // kNvlsUnroll switch reductions in flight per thread before the first is used (their
  // round trip through the NVSwitch is the latency to cover)
  const long long stride = 8ll * (long long)gridDim.x * blockDim.x;
  for (long long i0 = lo + 8ll * ((long long)blockIdx.x * blockDim.x + threadIdx.x); i0 < hi;
       i0 += kNvlsUnroll * stride) {
    float g[kNvlsUnroll][8];
#pragma unroll
    for (int u = 0; u < kNvlsUnroll; ++u)
      if (i0 + u * stride < hi) mc_sum8(mc_grad + i0 + u * stride, g[u]);
#pragma unroll
    for (int u = 0; u < kNvlsUnroll; ++u) {
      const long long i = i0 + u * stride;
      if (i >= hi) break;
#pragma unroll
      for (int k = 0; k < 8; ++k) g[u][k] *= scale;
      adamw8_multicast(i, i - lo, g[u], mc_shadow, mc_master, master, m, v, lr, b1, b2, eps, wd, bc1, bc2);
    }
  }
}

template <typename GT>
__global__ void __launch_bounds__(256) ddp_reduce_nvls_kernel(const GT* mc_grad, float inv_world, long long lo,
                                                              long long hi, float* __restrict__ gred,
                                                              float* __restrict__ sumsq) {
  float acc = 0.f;
  const long long stride = 8ll * (long long)gridDim.x * blockDim.x;
  for (long long i0 = lo + 8ll * ((long long)blockIdx.x * blockDim.x + threadIdx.x); i0 < hi;
       i0 += kNvlsUnroll * stride) {
    float g[kNvlsUnroll][8];
#pragma unroll
    for (int u = 0; u < kNvlsUnroll; ++u)
      if (i0 + u * stride < hi) mc_sum8(mc_grad + i0 + u * stride, g[u]);
#pragma unroll
    for (int u = 0; u < kNvlsUnroll; ++u) {
      const long long i = i0 + u * stride;
      if (i >= hi) break;
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        g[u][k] *= inv_world;
        acc += g[u][k] * g[u][k];
      }
      float* o = gred + (i - lo);
      *reinterpret_cast<float4*>(o) = make_float4(g[u][0], g[u][1], g[u][2], g[u][3]);
      *reinterpret_cast<float4*>(o + 4) = make_float4(g[u][4], g[u][5], g[u][6], g[u][7]);
    }
  }
  const float t = block_sum(acc);
  if (threadIdx.x == 0) atomicAdd(sumsq, t);
}

__global__ void __launch_bounds__(256) ddp_apply_nvls_kernel(__nv_bfloat16* mc_shadow, float* mc_master, long long lo,
                                                             long long hi, const float* __restrict__ gred,
                                                             float* __restrict__ master, float* __restrict__ m,
                                                             float* __restrict__ v, float b1, float b2, float eps,
                                                             float wd, const float* __restrict__ hyper,
                                                             const float* __restrict__ coef) {
  const float lr = hyper[0], bc1 = hyper[1], bc2 = hyper[2];
  const float c = coef[0];
  for (long long i = lo + 8ll * ((long long)blockIdx.x * blockDim.x + threadIdx.x); i < hi;
       i += 8ll * (long long)gridDim.x * blockDim.x) {
    float g[8];
    Vec8<float>::load(gred + (i - lo), g);
#pragma unroll
    for (int k = 0; k < 8; ++k) g[k] *= c;
    adamw8_multicast(i, i - lo, g, mc_shadow, mc_master, master, m, v, lr, b1, b2, eps, wd, bc1, bc2);
  }
}

// Flag page of the data-parallel step (DDP_FLAG_WORDS words per rank, symmetric): slot s
// of the per-bucket barriers uses words [8 s, 8 s + 8) (one word per source rank), the
// norm exchange its flag words at kDdpNormFlag and values at kDdpNormVal, and
// kDdpEpoch holds this rank's step counter (ddp_epoch_advance, once per step).
constexpr int kDdpNormFlag = 480;
constexpr int kDdpNormVal = 488;
constexpr int kDdpEpoch = 500;
constexpr int kDdpSlots = 60;

// Global gradient norm across the ranks: each rank publishes its sum of squares into
// every peer's flag page (value, then an epoch flag with release semantics), waits
// (bounded) for all W values of this step's epoch, and writes {clip coefficient, norm}
// to out.
__global__ void ddp_norm_exchange_kernel(PeerPtrs pp, int rank, int world, const float* __restrict__ sumsq,
                                         float max_norm, float* __restrict__ out, int* err) {
  const int t = threadIdx.x;
  __shared__ float vals[kMaxRanks];
  const unsigned int epoch = *(volatile unsigned int*)(pp.flags[rank] + kDdpEpoch);
  const float mine = *sumsq;
  if (t < world) {
    pp.flags[t][kDdpNormVal + rank] = __float_as_uint(mine);
    __threadfence_system();
    st_release_sys(pp.flags[t] + kDdpNormFlag + rank, epoch);
    const unsigned long long t0 = gtimer();
    float val = 0.f;
    while (true) {
      if (ld_acquire_sys(pp.flags[rank] + kDdpNormFlag + t) >= epoch) {
        val = __uint_as_float(*(volatile unsigned int*)(pp.flags[rank] + kDdpNormVal + t));
        break;
      }
      if (gtimer() - t0 > kPeerWaitNs) {
        atomicCAS(err, 0, 110);
        break;
      }
    }
    vals[t] = val;
  }
  __syncthreads();
  if (t == 0) {
    float tot = 0.f;
    for (int r = 0; r < world; ++r) tot += vals[r];
    const float norm = sqrtf(tot);
    out[0] = fminf(1.0f, max_norm / (norm + 1e-6f));
    out[1] = norm;
  }
}

// Advance this rank's step epoch (one thread; ordered before the step's barriers by the
// stream, or by the event the side stream waits on).
__global__ void ddp_epoch_advance_kernel(unsigned int* flags_local) { flags_local[kDdpEpoch] += 1; }

// Barrier of slot `slot` for this step's epoch: release-store the epoch into every peer's
// word [8 slot + rank], then wait (bounded, error code 120 + slot) until every peer has
// stored it into ours. Orders this rank's earlier writes (its bf16 gradients) before the
// peers' loads, and the peers' writes before ours.
__global__ void ddp_slot_barrier_kernel(PeerPtrs pp, int rank, int world, int slot, int* err) {
  const int t = threadIdx.x;
  const unsigned int epoch = *(volatile unsigned int*)(pp.flags[rank] + kDdpEpoch);
  __threadfence_system();
  __syncwarp();
  if (t < world) st_release_sys(pp.flags[t] + 8 * slot + rank, epoch);
  if (t < world) {
    const unsigned int* mine = pp.flags[rank] + 8 * slot + t;
    const unsigned long long t0 = gtimer();
    while (ld_acquire_sys(mine) < epoch) {
      if (gtimer() - t0 > kPeerWaitNs) {
        atomicCAS(err, 0, 120 + slot);
        break;
      }
    }
  }
  __syncwarp();
}


// Sequence-parallel halves of the tensor-parallel sums. tp_sum_slots: the owner adds its
// W slots (rows scattered to it by every rank) into its own rows, without gathering them.
__global__ void tp_sum_slots_kernel(const float* __restrict__ slots, float* __restrict__ out, int world,
                                    long long n4, long long slot_stride, const float* __restrict__ add) {
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (long long)gridDim.x * blockDim.x) {
    const long long e = 4 * i;
    float4 acc = add ? *reinterpret_cast<const float4*>(add + e) : make_float4(0.f, 0.f, 0.f, 0.f);
    for (int s = 0; s < world; ++s) {
      const float4 x = *reinterpret_cast<const float4*>(slots + s * slot_stride + e);
      acc.x += x.x;
      acc.y += x.y;
      acc.z += x.z;
      acc.w += x.w;
    }
    *reinterpret_cast<float4*>(out + e) = acc;
  }
}

// tp_gather_bytes: this rank's block of `nbytes` (16-byte multiples) at `offset` of its
// own buffer is stored at the same offset of every peer's buffer (an all-gather by P2P
// stores; the bf16 residual rows of sequence parallelism).
__global__ void tp_gather_bytes_kernel(const uint4* __restrict__ src, DstPtrs dp, int world, int rank,
                                       long long offset16, long long n16) {
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n16; i += (long long)gridDim.x * blockDim.x) {
    const uint4 x = src[offset16 + i];
    for (int r = 1; r < world; ++r) {
      int t = rank + r;
      if (t >= world) t -= world;
      reinterpret_cast<uint4*>(dp.dst[t])[offset16 + i] = x;
    }
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


namespace {
DdpPtrs make_ddp_ptrs(const std::vector<int64_t>& grad, const std::vector<int64_t>& shadow,
                      const std::vector<int64_t>& master = {}) {
  DdpPtrs pp;
  memset(&pp, 0, sizeof(pp));
  TORCH_CHECK(grad.size() >= 1 && grad.size() <= kMaxRanks && shadow.size() == grad.size(),
              "one gradient and one shadow pointer per rank (<= 8)");
  TORCH_CHECK(master.empty() || master.size() == grad.size(), "one master pointer per rank, or none");
  for (size_t r = 0; r < grad.size(); ++r) {
    pp.grad[r] = reinterpret_cast<const void*>(grad[r]);
    pp.shadow[r] = reinterpret_cast<__nv_bfloat16*>(shadow[r]);
    if (!master.empty()) pp.master[r] = reinterpret_cast<float*>(master[r]);
    TORCH_CHECK(grad[r] % 16 == 0 && shadow[r] % 16 == 0, "peer buffers must be 16-byte aligned");
  }
  return pp;
}

template <typename F>
void dispatch_world(int world, F&& f) {
  switch (world) {
    case 1: f(std::integral_constant<int, 1>{}); break;
    case 2: f(std::integral_constant<int, 2>{}); break;
    case 3: f(std::integral_constant<int, 3>{}); break;
    case 4: f(std::integral_constant<int, 4>{}); break;
    case 5: f(std::integral_constant<int, 5>{}); break;
    case 6: f(std::integral_constant<int, 6>{}); break;
    case 7: f(std::integral_constant<int, 7>{}); break;
    case 8: f(std::integral_constant<int, 8>{}); break;
    default: TORCH_CHECK(false, "1..8 ranks");
  }
}

int ddp_grid(long long n8) {
  // enough 8-element work items in flight to cover NVLink latency, never more blocks
  // than work
  const long long blocks = (n8 + 255) / 256;
  return (int)std::max<long long>(1, std::min<long long>(blocks, 148 * 4));
}
}  // namespace

// One fused data-parallel optimizer step (no clipping): see ddp_step_kernel.
// gather_master: every rank's fp32 master buffer (symmetric) to all-gather the new fp32
// values into as well, or empty.
void ddp_step(std::vector<int64_t> grad, std::vector<int64_t> shadow, bool grad_bf16, int64_t rank, int64_t lo,
              int64_t hi, const at::Tensor& master, const at::Tensor& m, const at::Tensor& v, double b1, double b2,
              double eps, double wd, const at::Tensor& hyper, const c10::optional<at::Tensor>& coef,
              std::vector<int64_t> gather_master) {
  DdpPtrs pp = make_ddp_ptrs(grad, shadow, gather_master);
  TORCH_CHECK(lo % 8 == 0 && hi % 8 == 0 && hi >= lo, "shard bounds must be multiples of 8");
  TORCH_CHECK(master.scalar_type() == at::kFloat && master.numel() >= hi, "fp32 master covering the shard");
  TORCH_CHECK(m.numel() >= hi - lo && v.numel() >= hi - lo, "moment shards too small");
  auto st = at::cuda::getCurrentCUDAStream(m.get_device()).stream();
  const int grid = ddp_grid((hi - lo) / 8);
  const float* cp = coef ? coef->data_ptr<float>() : nullptr;
  dispatch_world((int)grad.size(), [&](auto W) {
    if (grad_bf16)
      ddp_step_kernel<W(), __nv_bfloat16><<<grid, 256, 0, st>>>(
          pp, (int)rank, lo, hi, master.data_ptr<float>(), m.data_ptr<float>(), v.data_ptr<float>(), (float)b1,
          (float)b2, (float)eps, (float)wd, hyper.data_ptr<float>(), cp);
    else
      ddp_step_kernel<W(), float><<<grid, 256, 0, st>>>(pp, (int)rank, lo, hi, master.data_ptr<float>(),
                                                        m.data_ptr<float>(), v.data_ptr<float>(), (float)b1,
                                                        (float)b2, (float)eps, (float)wd, hyper.data_ptr<float>(), cp);
  });
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Clipping pass 1: peer sum of the owned slice into gred, its sum of squares into sumsq[0].
void ddp_reduce(std::vector<int64_t> grad, std::vector<int64_t> shadow, bool grad_bf16, int64_t rank, int64_t lo,
                int64_t hi, const at::Tensor& gred, const at::Tensor& sumsq) {
  DdpPtrs pp = make_ddp_ptrs(grad, shadow);
  TORCH_CHECK(lo % 8 == 0 && hi % 8 == 0 && gred.numel() >= hi - lo, "shard bounds / reduced shard size");
  auto st = at::cuda::getCurrentCUDAStream(gred.get_device()).stream();
  C10_CUDA_CHECK(cudaMemsetAsync(sumsq.data_ptr<float>(), 0, sizeof(float), st));
  const int grid = ddp_grid((hi - lo) / 8);
  dispatch_world((int)grad.size(), [&](auto W) {
    if (grad_bf16)
      ddp_reduce_kernel<W(), __nv_bfloat16><<<grid, 256, 0, st>>>(pp, (int)rank, lo, hi, gred.data_ptr<float>(),
                                                                  sumsq.data_ptr<float>());
    else
      ddp_reduce_kernel<W(), float><<<grid, 256, 0, st>>>(pp, (int)rank, lo, hi, gred.data_ptr<float>(),
                                                          sumsq.data_ptr<float>());
  });
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Clipping pass 2: AdamW from the reduced shard scaled by coef[0], shadow all-gather.
void ddp_apply(std::vector<int64_t> grad, std::vector<int64_t> shadow, int64_t rank, int64_t lo, int64_t hi,
               const at::Tensor& gred, const at::Tensor& master, const at::Tensor& m, const at::Tensor& v, double b1,
               double b2, double eps, double wd, const at::Tensor& hyper, const at::Tensor& coef,
               std::vector<int64_t> gather_master) {
  DdpPtrs pp = make_ddp_ptrs(grad, shadow, gather_master);
  TORCH_CHECK(lo % 8 == 0 && hi % 8 == 0 && gred.numel() >= hi - lo, "shard bounds / reduced shard size");
  auto st = at::cuda::getCurrentCUDAStream(gred.get_device()).stream();
  const int grid = ddp_grid((hi - lo) / 8);
  dispatch_world((int)grad.size(), [&](auto W) {
    ddp_apply_kernel<W()><<<grid, 256, 0, st>>>(pp, (int)rank, lo, hi, gred.data_ptr<float>(),
                                                master.data_ptr<float>(), m.data_ptr<float>(), v.data_ptr<float>(),
                                                (float)b1, (float)b2, (float)eps, (float)wd, hyper.data_ptr<float>(),
                                                coef.data_ptr<float>());
  });
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void ddp_epoch_advance(const at::Tensor& flags_local) {
  TORCH_CHECK(flags_local.numel() > kDdpEpoch, "flag page too small");
  auto st = at::cuda::getCurrentCUDAStream(flags_local.get_device()).stream();
  ddp_epoch_advance_kernel<<<1, 1, 0, st>>>(reinterpret_cast<unsigned int*>(flags_local.data_ptr()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void ddp_slot_barrier(std::vector<int64_t> flags, int64_t rank, int64_t slot, const at::Tensor& err) {
  TORCH_CHECK(slot >= 0 && slot < kDdpSlots, "barrier slot out of range");
  std::vector<int64_t> z(flags.size(), 0);
  PeerPtrs pp = make_ptrs(z, z, z, flags);
  auto st = at::cuda::getCurrentCUDAStream(err.get_device()).stream();
  ddp_slot_barrier_kernel<<<1, 32, 0, st>>>(pp, (int)rank, (int)flags.size(), (int)slot, err.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Cross-rank global norm: see ddp_norm_exchange_kernel. out = {coef, norm}.
void ddp_norm_exchange(std::vector<int64_t> flags, int64_t rank, const at::Tensor& sumsq, double max_norm,
                       const at::Tensor& out, const at::Tensor& err) {
  std::vector<int64_t> z(flags.size(), 0);
  PeerPtrs pp = make_ptrs(z, z, z, flags);
  auto st = at::cuda::getCurrentCUDAStream(out.get_device()).stream();
  ddp_norm_exchange_kernel<<<1, 32, 0, st>>>(pp, (int)rank, (int)flags.size(), sumsq.data_ptr<float>(),
                                             (float)max_norm, out.data_ptr<float>(), err.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}


// out[e] = (add[e]) + sum_s slots[s * slot_stride + e] for e < n (n % 4 == 0)
void tp_sum_slots(const at::Tensor& slots, const at::Tensor& out, int64_t world, int64_t n, int64_t slot_stride,
                  const c10::optional<at::Tensor>& add) {
  TORCH_CHECK(n % 4 == 0 && slot_stride % 4 == 0 && out.numel() >= n, "tp_sum_slots: sizes");
  auto st = at::cuda::getCurrentCUDAStream(out.get_device()).stream();
  tp_sum_slots_kernel<<<148 * 2, 256, 0, st>>>(slots.data_ptr<float>(), out.data_ptr<float>(), (int)world, n / 4,
                                               slot_stride, add ? add->data_ptr<float>() : nullptr);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Store bytes [offset, offset + nbytes) of this rank's buffer (dst[rank]) into every peer's.
void tp_gather_bytes(std::vector<int64_t> dst, int64_t rank, int64_t offset, int64_t nbytes, int64_t device) {
  const int world = (int)dst.size();
  TORCH_CHECK(world >= 1 && world <= kMaxRanks && offset % 16 == 0 && nbytes % 16 == 0, "tp_gather_bytes: 16-byte blocks");
  DstPtrs dp;
  memset(&dp, 0, sizeof(dp));
  for (int r = 0; r < world; ++r) dp.dst[r] = reinterpret_cast<float*>(dst[r]);
  auto st = at::cuda::getCurrentCUDAStream((c10::DeviceIndex)device).stream();
  tp_gather_bytes_kernel<<<148 * 2, 256, 0, st>>>(reinterpret_cast<const uint4*>(dst[rank]), dp, world, (int)rank,
                                                  offset / 16, nbytes / 16);
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


// NVLS forms of ddp_step / ddp_reduce / ddp_apply: mc_* are multicast addresses of the
// gradient, shadow and (0: not gathered) master buffers; the rest as in the P2P forms.
void ddp_step_nvls(int64_t mc_grad, int64_t mc_shadow, int64_t mc_master, bool grad_bf16, int64_t world, int64_t lo,
                   int64_t hi, const at::Tensor& master, const at::Tensor& m, const at::Tensor& v, double b1,
                   double b2, double eps, double wd, const at::Tensor& hyper, const c10::optional<at::Tensor>& coef) {
  TORCH_CHECK(mc_grad != 0 && mc_shadow != 0, "multicast addresses of the gradient and shadow buffers");
  TORCH_CHECK(lo % 8 == 0 && hi % 8 == 0 && hi >= lo && world >= 1, "shard bounds must be multiples of 8");
  TORCH_CHECK(master.scalar_type() == at::kFloat && master.numel() >= hi, "fp32 master covering the shard");
  TORCH_CHECK(m.numel() >= hi - lo && v.numel() >= hi - lo, "moment shards too small");
  auto st = at::cuda::getCurrentCUDAStream(m.get_device()).stream();
  const int grid = ddp_grid((hi - lo) / 8);
  const float* cp = coef ? coef->data_ptr<float>() : nullptr;
  auto* sh = reinterpret_cast<__nv_bfloat16*>(mc_shadow);
  auto* mm = reinterpret_cast<float*>(mc_master);
  if (grad_bf16)
    ddp_step_nvls_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(
        reinterpret_cast<const __nv_bfloat16*>(mc_grad), sh, mm, 1.0f / (float)world, lo, hi, master.data_ptr<float>(),
        m.data_ptr<float>(), v.data_ptr<float>(), (float)b1, (float)b2, (float)eps, (float)wd, hyper.data_ptr<float>(),
        cp);
  else
    ddp_step_nvls_kernel<float><<<grid, 256, 0, st>>>(
        reinterpret_cast<const float*>(mc_grad), sh, mm, 1.0f / (float)world, lo, hi, master.data_ptr<float>(),
        m.data_ptr<float>(), v.data_ptr<float>(), (float)b1, (float)b2, (float)eps, (float)wd, hyper.data_ptr<float>(),
        cp);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void ddp_reduce_nvls(int64_t mc_grad, bool grad_bf16, int64_t world, int64_t lo, int64_t hi, const at::Tensor& gred,
                     const at::Tensor& sumsq) {
  TORCH_CHECK(mc_grad != 0 && lo % 8 == 0 && hi % 8 == 0 && gred.numel() >= hi - lo, "shard bounds / reduced shard");
  auto st = at::cuda::getCurrentCUDAStream(gred.get_device()).stream();
  C10_CUDA_CHECK(cudaMemsetAsync(sumsq.data_ptr<float>(), 0, sizeof(float), st));
  const int grid = ddp_grid((hi - lo) / 8);
  if (grad_bf16)
    ddp_reduce_nvls_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(reinterpret_cast<const __nv_bfloat16*>(mc_grad),
                                                                1.0f / (float)world, lo, hi, gred.data_ptr<float>(),
                                                                sumsq.data_ptr<float>());
  else
    ddp_reduce_nvls_kernel<float><<<grid, 256, 0, st>>>(reinterpret_cast<const float*>(mc_grad), 1.0f / (float)world,
                                                        lo, hi, gred.data_ptr<float>(), sumsq.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void ddp_apply_nvls(int64_t mc_shadow, int64_t mc_master, int64_t lo, int64_t hi, const at::Tensor& gred,
                    const at::Tensor& master, const at::Tensor& m, const at::Tensor& v, double b1, double b2,
                    double eps, double wd, const at::Tensor& hyper, const at::Tensor& coef) {
  TORCH_CHECK(mc_shadow != 0 && lo % 8 == 0 && hi % 8 == 0, "multicast shadow address / shard bounds");
  auto st = at::cuda::getCurrentCUDAStream(m.get_device()).stream();
  const int grid = ddp_grid((hi - lo) / 8);
  ddp_apply_nvls_kernel<<<grid, 256, 0, st>>>(reinterpret_cast<__nv_bfloat16*>(mc_shadow),
                                              reinterpret_cast<float*>(mc_master), lo, hi, gred.data_ptr<float>(),
                                              master.data_ptr<float>(), m.data_ptr<float>(), v.data_ptr<float>(),
                                              (float)b1, (float)b2, (float)eps, (float)wd, hyper.data_ptr<float>(),
                                              coef.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace bd
