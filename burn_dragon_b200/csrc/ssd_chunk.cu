// ssd_chunk.cu — the chunked state-space-duality scan of the Mamba-3 memory, forward and
// backward, one CTA per (batch, head) walking its chunks in order (forward) or in
// reverse (backward) with the state held in shared memory.
//
// Per chunk c of C tokens (q, k [C, S] rotated / scaled keys and queries, v [C, P], da [C]
// the chunk-local cumulative log decay, cf / vs / ks the trapezoid term that enters at
// the chunk boundary), with S the state [P, S] entering the chunk:
//   tilde  = S + cf * vs ks^T
//   y_i    = e^{da_i} tilde q_i + sum_{j<i} (q_i . k_j) e^{min(da_i - da_j, 0)} v_j
//   S'     = e^{da_last} tilde + sum_j e^{da_last - da_j} v_j k_j^T
// (burn_dragon_kernel/src/sequence/mamba3/forward.rs:1738-2346; the PyTorch restatement
// is models/sequence.py Mamba3Params.forward). The forward keeps every chunk's tilde for
// the backward, which carries dS' back through the chunks and produces the gradients of
// q, k, v, da, the initial state and the trapezoid inputs.
//
// All products are fp32 on the CUDA cores: the per-head operands are small (C <= 64,
// S <= 64, P <= 128; Mamba-3's defaults are C = 64, S = 16, P = 128), and the scan is
// sequential over chunks, so the cost is the chunk loop, which this kernel runs without
// a launch per chunk.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

namespace bd {
namespace {

constexpr int kThreads = 256;

struct SsdDims {
  int T, C, S, P, n;  // tokens, chunk, state, head dim, chunks
};

// shared-memory carve-up, the same in forward and backward (floats)
struct SsdSmem {
  float *st, *tl, *q, *k, *v, *da, *ex, *wx, *A, *QK, *dy, *dst, *dtl, *U, *V2, *red;
};

__device__ __forceinline__ SsdSmem carve(float* base, const SsdDims& d, bool bwd) {
  SsdSmem m;
  float* p = base;
  m.st = p; p += d.P * d.S;    // state (forward) / dS (backward)
  m.tl = p; p += d.P * d.S;    // tilde
  m.q = p; p += d.C * d.S;
  m.k = p; p += d.C * d.S;
  m.v = p; p += d.C * d.P;
  m.da = p; p += 64;
  m.ex = p; p += 64;           // e^{da_i}
  m.wx = p; p += 64;           // e^{da_last - da_j}
  m.A = p; p += d.C * d.C;     // (q.k) L, masked
  m.QK = p; p += d.C * d.C;    // q.k (backward: the decay gradient needs it)
  m.dy = bwd ? p : nullptr; if (bwd) p += d.C * d.P;
  m.dst = bwd ? p : nullptr; if (bwd) p += d.C * d.C;  // dA
  m.dtl = bwd ? p : nullptr; if (bwd) p += d.P * d.S;  // dtilde
  m.U = bwd ? p : nullptr; if (bwd) p += d.C * d.S;    // U_i = tilde^T dy_i
  m.V2 = bwd ? p : nullptr; if (bwd) p += d.C * d.P;   // V2_j = dS' k_j
  m.red = p; p += 4 * 64;      // small reductions
  return m;
}

size_t smem_floats(const SsdDims& d, bool bwd) {
  size_t f = 2 * d.P * d.S + 2 * d.C * d.S + d.C * d.P + 3 * 64 + 2 * d.C * d.C + 4 * 64;
  if (bwd) f += d.C * d.P + d.C * d.C + d.P * d.S + d.C * d.S + d.C * d.P;
  return f;
}

// A[i][j] = j < i ? (q_i . k_j) exp(min(da_i - da_j, 0)) : 0, QK[i][j] = q_i . k_j
__device__ void chunk_scores(const SsdSmem& m, const SsdDims& d, int Cc) {
  for (int idx = threadIdx.x; idx < Cc * Cc; idx += kThreads) {
    const int i = idx / Cc, j = idx % Cc;
    float s = 0.f;
    if (j < i)
      for (int t = 0; t < d.S; ++t) s += m.q[i * d.S + t] * m.k[j * d.S + t];
    m.QK[i * d.C + j] = s;
    m.A[i * d.C + j] = j < i ? s * __expf(fminf(m.da[i] - m.da[j], 0.f)) : 0.f;
  }
}

__device__ void load_chunk(const SsdSmem& m, const SsdDims& d, int Cc, const float* q, const float* k,
                           const float* v, const float* da, long long t0) {
  for (int idx = threadIdx.x; idx < Cc * d.S; idx += kThreads) {
    m.q[idx] = q[t0 * d.S + idx];
    m.k[idx] = k[t0 * d.S + idx];
  }
  for (int idx = threadIdx.x; idx < Cc * d.P; idx += kThreads) m.v[idx] = v[t0 * d.P + idx];
  for (int idx = threadIdx.x; idx < Cc; idx += kThreads) m.da[idx] = da[t0 + idx];
}

// after load_chunk and a barrier: the per-token exponentials of the chunk
__device__ void chunk_exps(const SsdSmem& m, int Cc) {
  const float last = m.da[Cc - 1];
  for (int i = threadIdx.x; i < Cc; i += kThreads) {
    m.ex[i] = __expf(m.da[i]);
    m.wx[i] = __expf(last - m.da[i]);
  }
}

__global__ void __launch_bounds__(kThreads) ssd_fwd_kernel(SsdDims d, const float* __restrict__ Q,
                                                           const float* __restrict__ K, const float* __restrict__ V,
                                                           const float* __restrict__ DA, const float* __restrict__ S0,
                                                           const float* __restrict__ VS, const float* __restrict__ KS,
                                                           const float* __restrict__ CF, float* __restrict__ Y,
                                                           float* __restrict__ SF, float* __restrict__ SC) {
  extern __shared__ float sm[];
  const SsdSmem m = carve(sm, d, false);
  const long long bh = blockIdx.x;
  const float* q = Q + bh * d.T * d.S;
  const float* k = K + bh * d.T * d.S;
  const float* v = V + bh * d.T * d.P;
  const float* da = DA + bh * d.T;
  const int PS = d.P * d.S;
  for (int idx = threadIdx.x; idx < PS; idx += kThreads) m.st[idx] = S0[bh * PS + idx];
  for (int c = 0; c < d.n; ++c) {
    const long long t0 = (long long)c * d.C;
    const int Cc = min(d.C, d.T - (int)t0);
    __syncthreads();
    load_chunk(m, d, Cc, q, k, v, da, t0);
    const float cf = CF[bh * d.n + c];
    const float* vs = VS + (bh * d.n + c) * d.P;
    const float* ks = KS + (bh * d.n + c) * d.S;
    __syncthreads();
    chunk_exps(m, Cc);
    for (int idx = threadIdx.x; idx < PS; idx += kThreads) {
      const int p = idx / d.S, s = idx % d.S;
      const float tl = m.st[idx] + cf * vs[p] * ks[s];
      m.tl[idx] = tl;
      SC[(bh * d.n + c) * PS + idx] = tl;
    }
    __syncthreads();
    chunk_scores(m, d, Cc);
    __syncthreads();
    // y_i = e^{da_i} tilde q_i + sum_j A_ij v_j
    float* y = Y + (bh * d.T + t0) * d.P;
    for (int idx = threadIdx.x; idx < Cc * d.P; idx += kThreads) {
      const int i = idx / d.P, p = idx % d.P;
      float a = 0.f;
      for (int s = 0; s < d.S; ++s) a += m.tl[p * d.S + s] * m.q[i * d.S + s];
      a *= m.ex[i];
      for (int j = 0; j < i; ++j) a += m.A[i * d.C + j] * m.v[j * d.P + p];
      y[idx] = a;
    }
    // S' = e^{da_last} tilde + sum_j e^{da_last - da_j} v_j k_j^T
    const float last = m.da[Cc - 1];
    const float E = __expf(last);
    for (int idx = threadIdx.x; idx < PS; idx += kThreads) {
      const int p = idx / d.S, s = idx % d.S;
      float a = E * m.tl[idx];
      for (int j = 0; j < Cc; ++j) a += m.wx[j] * m.v[j * d.P + p] * m.k[j * d.S + s];
      m.st[idx] = a;
    }
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < PS; idx += kThreads) SF[bh * PS + idx] = m.st[idx];
}

// block-wide sum of one value per thread; valid in every thread after the call
__device__ float block_total(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = v;
  __syncthreads();
  float t = 0.f;
  for (int w = 0; w < kThreads / 32; ++w) t += red[w];
  __syncthreads();
  return t;
}

__global__ void __launch_bounds__(kThreads) ssd_bwd_kernel(
    SsdDims d, const float* __restrict__ Q, const float* __restrict__ K, const float* __restrict__ V,
    const float* __restrict__ DA, const float* __restrict__ VS, const float* __restrict__ KS,
    const float* __restrict__ CF, const float* __restrict__ SC, const float* __restrict__ DY,
    const float* __restrict__ DSF, float* __restrict__ dQ, float* __restrict__ dK, float* __restrict__ dV,
    float* __restrict__ dDA, float* __restrict__ dS0, float* __restrict__ dVS, float* __restrict__ dKS,
    float* __restrict__ dCF) {
  extern __shared__ float sm[];
  const SsdSmem m = carve(sm, d, true);
  const long long bh = blockIdx.x;
  const float* q = Q + bh * d.T * d.S;
  const float* k = K + bh * d.T * d.S;
  const float* v = V + bh * d.T * d.P;
  const float* da = DA + bh * d.T;
  const int PS = d.P * d.S;
  for (int idx = threadIdx.x; idx < PS; idx += kThreads) m.st[idx] = DSF[bh * PS + idx];  // dS'
  for (int c = d.n - 1; c >= 0; --c) {
    const long long t0 = (long long)c * d.C;
    const int Cc = min(d.C, d.T - (int)t0);
    __syncthreads();
    load_chunk(m, d, Cc, q, k, v, da, t0);
    const float* dy = DY + (bh * d.T + t0) * d.P;
    for (int idx = threadIdx.x; idx < Cc * d.P; idx += kThreads) m.dy[idx] = dy[idx];
    for (int idx = threadIdx.x; idx < PS; idx += kThreads) m.tl[idx] = SC[(bh * d.n + c) * PS + idx];
    __syncthreads();
    chunk_exps(m, Cc);
    chunk_scores(m, d, Cc);
    // DAL_ij = (dy_i . v_j) L_ij (j < i): the gradient of A_ij times its decay
    for (int idx = threadIdx.x; idx < Cc * Cc; idx += kThreads) {
      const int i = idx / Cc, j = idx % Cc;
      float s = 0.f;
      if (j < i) {
        for (int p = 0; p < d.P; ++p) s += m.dy[i * d.P + p] * m.v[j * d.P + p];
        s *= __expf(fminf(m.da[i] - m.da[j], 0.f));
      }
      m.dst[i * d.C + j] = s;
    }
    __syncthreads();
    const float last = m.da[Cc - 1];
    const float E = __expf(last);
    // dtilde = E dS' + sum_i e^{da_i} dy_i q_i^T
    for (int idx = threadIdx.x; idx < PS; idx += kThreads) {
      const int p = idx / d.S, s = idx % d.S;
      float a = E * m.st[idx];
      for (int i = 0; i < Cc; ++i) a += m.ex[i] * m.dy[i * d.P + p] * m.q[i * d.S + s];
      m.dtl[idx] = a;
    }
    __syncthreads();
    float* gq = dQ + (bh * d.T + t0) * d.S;
    float* gk = dK + (bh * d.T + t0) * d.S;
    float* gv = dV + (bh * d.T + t0) * d.P;
    float* gda = dDA + bh * d.T + t0;
    // dq_i = e^{da_i} tilde^T dy_i + sum_{j<i} dA_ij L_ij k_j
    for (int idx = threadIdx.x; idx < Cc * d.S; idx += kThreads) {
      const int i = idx / d.S, s = idx % d.S;
      float a = 0.f;
      for (int p = 0; p < d.P; ++p) a += m.tl[p * d.S + s] * m.dy[i * d.P + p];
      m.U[idx] = a;
      a *= m.ex[i];
      for (int j = 0; j < i; ++j) a += m.dst[i * d.C + j] * m.k[j * d.S + s];
      gq[idx] = a;
    }
    // dk_j = sum_{i>j} dA_ij L_ij q_i + w_j dS'^T v_j
    for (int idx = threadIdx.x; idx < Cc * d.S; idx += kThreads) {
      const int j = idx / d.S, s = idx % d.S;
      float a = 0.f;
      for (int i = j + 1; i < Cc; ++i) a += m.dst[i * d.C + j] * m.q[i * d.S + s];
      float b = 0.f;
      for (int p = 0; p < d.P; ++p) b += m.st[p * d.S + s] * m.v[j * d.P + p];
      gk[idx] = a + m.wx[j] * b;
    }
    // dv_j = sum_{i>j} A_ij dy_i + w_j dS' k_j
    for (int idx = threadIdx.x; idx < Cc * d.P; idx += kThreads) {
      const int j = idx / d.P, p = idx % d.P;
      float a = 0.f;
      for (int i = j + 1; i < Cc; ++i) a += m.A[i * d.C + j] * m.dy[i * d.P + p];
      float b = 0.f;
      for (int s = 0; s < d.S; ++s) b += m.st[p * d.S + s] * m.k[j * d.S + s];
      m.V2[idx] = b;
      gv[idx] = a + m.wx[j] * b;
    }
    __syncthreads();
    // decay gradient, per token (thread i < Cc), plus the chunk-last terms
    float extra_last = 0.f;
    if ((int)threadIdx.x < Cc) {
      const int i = threadIdx.x;
      const float ei = m.ex[i];
      // e^{da_i} dy_i . (tilde q_i) = e^{da_i} U_i . q_i
      float t1 = 0.f;
      for (int s = 0; s < d.S; ++s) t1 += m.U[i * d.S + s] * m.q[i * d.S + s];
      float g = ei * t1;
      // intra-chunk decay: G_ij = dA_ij L_ij QK_ij where da_i - da_j <= 0
      for (int j = 0; j < i; ++j)
        if (m.da[i] - m.da[j] <= 0.f) g += m.dst[i * d.C + j] * m.QK[i * d.C + j];
      for (int i2 = i + 1; i2 < Cc; ++i2)
        if (m.da[i2] - m.da[i] <= 0.f) g -= m.dst[i2 * d.C + i] * m.QK[i2 * d.C + i];
      // state write: R_i = w_i v_i^T dS' k_i enters with -1 here and +1 on the last token
      float r = 0.f;
      for (int p = 0; p < d.P; ++p) r += m.v[i * d.P + p] * m.V2[i * d.P + p];
      r *= m.wx[i];
      g -= r;
      extra_last = r;
      gda[i] = g;
    }
    // + E <tilde, dS'> on the last token, and the sum of R
    float tds = 0.f;
    for (int idx = threadIdx.x; idx < PS; idx += kThreads) tds += m.tl[idx] * m.st[idx];
    const float tot = block_total(E * tds + extra_last, m.red);
    if (threadIdx.x == 0) gda[Cc - 1] += tot;
    // trapezoid inputs: tilde = S + cf vs ks^T
    const float cf = CF[bh * d.n + c];
    const float* vs = VS + (bh * d.n + c) * d.P;
    const float* ks = KS + (bh * d.n + c) * d.S;
    float dcf = 0.f;
    for (int idx = threadIdx.x; idx < PS; idx += kThreads) {
      const int p = idx / d.S, s = idx % d.S;
      dcf += m.dtl[idx] * vs[p] * ks[s];
    }
    const float dcf_tot = block_total(dcf, m.red);
    if (threadIdx.x == 0) dCF[bh * d.n + c] = dcf_tot;
    for (int p = threadIdx.x; p < d.P; p += kThreads) {
      float a = 0.f;
      for (int s = 0; s < d.S; ++s) a += m.dtl[p * d.S + s] * ks[s];
      dVS[(bh * d.n + c) * d.P + p] = cf * a;
    }
    for (int s = threadIdx.x; s < d.S; s += kThreads) {
      float a = 0.f;
      for (int p = 0; p < d.P; ++p) a += m.dtl[p * d.S + s] * vs[p];
      dKS[(bh * d.n + c) * d.S + s] = cf * a;
    }
    __syncthreads();
    // the gradient entering the previous chunk's output state
    for (int idx = threadIdx.x; idx < PS; idx += kThreads) m.st[idx] = m.dtl[idx];
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < PS; idx += kThreads) dS0[bh * PS + idx] = m.st[idx];
}

SsdDims dims_of(const at::Tensor& q, const at::Tensor& v, int64_t chunk) {
  SsdDims d;
  d.T = (int)q.size(1);
  d.S = (int)q.size(2);
  d.P = (int)v.size(2);
  d.C = (int)chunk;
  d.n = (d.T + d.C - 1) / d.C;
  TORCH_CHECK(d.C >= 1 && d.C <= 64 && d.S <= 64 && d.P <= 256, "ssd_chunk: chunk <= 64, state <= 64, head dim <= 256");
  return d;
}

void check_f32(std::initializer_list<const at::Tensor*> ts) {
  for (auto* t : ts) TORCH_CHECK(t->scalar_type() == at::kFloat && t->is_contiguous() && t->is_cuda(),
                                 "ssd_chunk: fp32 contiguous CUDA tensors");
}

}  // namespace

// Q, K [BH, T, S]; V [BH, T, P]; DA [BH, T]; S0 [BH, P, S]; VS [BH, n, P]; KS [BH, n, S];
// CF [BH, n] -> Y [BH, T, P], SF [BH, P, S], SC [BH, n, P, S] (every chunk's tilde).
void ssd_chunk_fwd(const at::Tensor& Q, const at::Tensor& K, const at::Tensor& V, const at::Tensor& DA,
                   const at::Tensor& S0, const at::Tensor& VS, const at::Tensor& KS, const at::Tensor& CF,
                   int64_t chunk, const at::Tensor& Y, const at::Tensor& SF, const at::Tensor& SC) {
  check_f32({&Q, &K, &V, &DA, &S0, &VS, &KS, &CF, &Y, &SF, &SC});
  const SsdDims d = dims_of(Q, V, chunk);
  TORCH_CHECK(SC.numel() == Q.size(0) * d.n * d.P * d.S && CF.numel() == Q.size(0) * d.n, "ssd_chunk: sizes");
  c10::cuda::CUDAGuard g(Q.get_device());
  const size_t bytes = smem_floats(d, false) * sizeof(float);
  TORCH_CHECK(bytes <= 227 * 1024, "ssd_chunk: chunk / state / head dims need too much shared memory");
  C10_CUDA_CHECK(cudaFuncSetAttribute(ssd_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes));
  ssd_fwd_kernel<<<(unsigned)Q.size(0), kThreads, bytes, at::cuda::getCurrentCUDAStream(Q.get_device()).stream()>>>(
      d, Q.data_ptr<float>(), K.data_ptr<float>(), V.data_ptr<float>(), DA.data_ptr<float>(), S0.data_ptr<float>(),
      VS.data_ptr<float>(), KS.data_ptr<float>(), CF.data_ptr<float>(), Y.data_ptr<float>(), SF.data_ptr<float>(),
      SC.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void ssd_chunk_bwd(const at::Tensor& Q, const at::Tensor& K, const at::Tensor& V, const at::Tensor& DA,
                   const at::Tensor& VS, const at::Tensor& KS, const at::Tensor& CF, const at::Tensor& SC,
                   const at::Tensor& DY, const at::Tensor& DSF, int64_t chunk, const at::Tensor& dQ,
                   const at::Tensor& dK, const at::Tensor& dV, const at::Tensor& dDA, const at::Tensor& dS0,
                   const at::Tensor& dVS, const at::Tensor& dKS, const at::Tensor& dCF) {
  check_f32({&Q, &K, &V, &DA, &VS, &KS, &CF, &SC, &DY, &DSF, &dQ, &dK, &dV, &dDA, &dS0, &dVS, &dKS, &dCF});
  const SsdDims d = dims_of(Q, V, chunk);
  c10::cuda::CUDAGuard g(Q.get_device());
  const size_t bytes = smem_floats(d, true) * sizeof(float);
  TORCH_CHECK(bytes <= 227 * 1024, "ssd_chunk: chunk / state / head dims need too much shared memory");
  C10_CUDA_CHECK(cudaFuncSetAttribute(ssd_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes));
  ssd_bwd_kernel<<<(unsigned)Q.size(0), kThreads, bytes, at::cuda::getCurrentCUDAStream(Q.get_device()).stream()>>>(
      d, Q.data_ptr<float>(), K.data_ptr<float>(), V.data_ptr<float>(), DA.data_ptr<float>(), VS.data_ptr<float>(),
      KS.data_ptr<float>(), CF.data_ptr<float>(), SC.data_ptr<float>(), DY.data_ptr<float>(), DSF.data_ptr<float>(),
      dQ.data_ptr<float>(), dK.data_ptr<float>(), dV.data_ptr<float>(), dDA.data_ptr<float>(), dS0.data_ptr<float>(),
      dVS.data_ptr<float>(), dKS.data_ptr<float>(), dCF.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace bd
