// rowwise.cu — memory-bound row kernels of the BDH step, one warp per row.
//
// LayerNorm here is the reference's shared `DragonNorm` (LayerNorm with gamma/beta,
// eps 1e-5; burn_dragon_core/src/model/norm.rs:302-327). Each lane holds D/32 values
// (lane-strided, so loads are coalesced); statistics are fp32.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_bf16.h>
#include <torch/extension.h>

namespace bd {
namespace {

constexpr int kWarps = 8;

// Bounds checks of the data-dependent indices (token ids, targets), on only while a debug
// word is registered for the device (set_debug_bounds; DRAGON_DEBUG_BOUNDS=1 at the Python
// layer): a token or target outside [0, V) records its code in the word (first one wins)
// and the access is skipped, so a bad batch is reported instead of faulting.
constexpr int kBoundsGather = 201;  // ln_fwd embedding gather: token id outside the table
constexpr int kBoundsTarget = 202;  // cross-entropy target outside the vocabulary
constexpr int kBoundsEmbedGrad = 203;  // embedding-gradient token id outside the table
int* g_debug_word[64] = {nullptr};

__device__ __forceinline__ bool in_vocab(int64_t t, long long V, int* dbg, int code) {
  if (dbg == nullptr || (t >= 0 && t < V)) return true;
  atomicCAS(dbg, 0, code);
  return false;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Normalisation kinds of the shared norm (burn_dragon_core/src/model/norm.rs:302-327),
// every one followed by y = n * gamma + beta:
//   0 LayerNorm    n = (x - mean) / sqrt(var + eps)
//   1 RMSNorm      n = x / sqrt(mean(x^2) + eps)
//   2 DynamicTanh  n = tanh(alpha x)
//   3 Derf         n = erf(alpha x + shift)
// alpha / shift are learnable scalars (device pointers). The statistics saved for the
// backward are (mean, rstd) for kinds 0 / 1 and unused (0, 1) for the elementwise kinds.
struct NormArgs {
  int kind;
  const float* alpha;
  const float* shift;
};

// Rows of the gamma / beta (/ alpha / shift) gradient partials: the elementwise kinds add
// per-column partials of the two scalar gradients (summed over the columns on the host).
__host__ __device__ __forceinline__ int norm_part_rows(int kind) { return kind >= 2 ? 4 : 2; }

template <int VPL>
__device__ __forceinline__ void norm_row(const float (&x)[VPL], int D, float eps, const NormArgs& na,
                                         float (&n)[VPL], float& mean, float& rstd) {
  if (na.kind <= 1) {
    float s = 0.f;
    if (na.kind == 0) {
#pragma unroll
      for (int i = 0; i < VPL; ++i) s += x[i];
      mean = warp_sum(s) / D;
    } else {
      mean = 0.f;
    }
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const float d = x[i] - mean;
      q += d * d;
    }
    rstd = rsqrtf(warp_sum(q) / D + eps);
#pragma unroll
    for (int i = 0; i < VPL; ++i) n[i] = (x[i] - mean) * rstd;
  } else {
    mean = 0.f;
    rstd = 1.f;
    const float a = *na.alpha;
    const float sh = na.kind == 3 ? *na.shift : 0.f;
#pragma unroll
    for (int i = 0; i < VPL; ++i) n[i] = na.kind == 2 ? tanhf(a * x[i]) : erff(fmaf(a, x[i], sh));
  }
}

// The normalised row again from the raw input and the saved statistics.
template <int VPL>
__device__ __forceinline__ void norm_row_saved(const float (&x)[VPL], float mean, float rstd, const NormArgs& na,
                                               float (&n)[VPL]) {
  if (na.kind <= 1) {
#pragma unroll
    for (int i = 0; i < VPL; ++i) n[i] = (x[i] - mean) * rstd;
  } else {
    const float a = *na.alpha;
    const float sh = na.kind == 3 ? *na.shift : 0.f;
#pragma unroll
    for (int i = 0; i < VPL; ++i) n[i] = na.kind == 2 ? tanhf(a * x[i]) : erff(fmaf(a, x[i], sh));
  }
}

// dx of y = n(x) * gamma + beta given dy = g (x raw, n its normalised row); accumulates the
// lane partials of dgamma / dbeta and, for the elementwise kinds, of dalpha / dshift.
template <int VPL>
__device__ __forceinline__ void norm_backward_row(const float (&g)[VPL], const float (&x)[VPL], const float (&n)[VPL],
                                                  const float (&gam)[VPL], float rstd, int D, const NormArgs& na,
                                                  float (&dx)[VPL], float (&dg)[VPL], float (&db)[VPL],
                                                  float (&da)[VPL], float (&ds)[VPL]) {
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    dg[i] += g[i] * n[i];
    db[i] += g[i];
  }
  if (na.kind <= 1) {
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const float gy = g[i] * gam[i];
      s1 += gy;
      s2 += gy * n[i];
    }
    s1 = na.kind == 0 ? warp_sum(s1) / D : 0.f;
    s2 = warp_sum(s2) / D;
#pragma unroll
    for (int i = 0; i < VPL; ++i) dx[i] = rstd * (g[i] * gam[i] - s1 - n[i] * s2);
  } else {
    const float a = *na.alpha;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const float gy = g[i] * gam[i];
      // d n / d(alpha x + shift): 1 - tanh^2, or (2 / sqrt(pi)) exp(-z^2)
      float dn;
      if (na.kind == 2) {
        dn = 1.f - n[i] * n[i];
      } else {
        const float z = fmaf(a, x[i], *na.shift);
        dn = 1.1283791670955126f * __expf(-z * z);
      }
      dx[i] = gy * dn * a;
      da[i] += gy * dn * x[i];
      ds[i] += na.kind == 3 ? gy * dn : 0.f;
    }
  }
}

// Reduce per-lane partials over the block's warps and write one partial block per CTA:
// part[block, 0, :] = dgamma, part[block, 1, :] = dbeta (and rows 2, 3 = per-column
// dalpha / dshift partials for the elementwise kinds).
template <int VPL>
__device__ void block_write_partials(const float (&dg)[VPL], const float (&db)[VPL], const float (&da)[VPL],
                                     const float (&ds)[VPL], int D, int kind, float* part) {
  extern __shared__ float sh[];  // [kWarps][rows][D]
  const int R = norm_part_rows(kind);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    sh[(warp * R + 0) * D + lane + 32 * i] = dg[i];
    sh[(warp * R + 1) * D + lane + 32 * i] = db[i];
    if (R == 4) {
      sh[(warp * R + 2) * D + lane + 32 * i] = da[i];
      sh[(warp * R + 3) * D + lane + 32 * i] = ds[i];
    }
  }
  __syncthreads();
  for (int c = threadIdx.x; c < R * D; c += blockDim.x) {
    const int which = c / D, col = c % D;
    float s = 0.f;
    for (int w = 0; w < kWarps; ++w) s += sh[(w * R + which) * D + col];
    part[(size_t)blockIdx.x * R * D + c] = s;
  }
}

// y = norm(x) for rows of x (fp32); optional fp32 / bf16 outputs and saved stats.
// When `tokens` is given the row is gathered from an embedding table first.
template <int VPL>
__global__ void ln_fwd_kernel(const float* __restrict__ x, const int64_t* __restrict__ tokens, long long rows, int D,
                              const float* __restrict__ gamma, const float* __restrict__ beta, float eps,
                              float* __restrict__ y32, __nv_bfloat16* __restrict__ y16, float* __restrict__ mean_out,
                              float* __restrict__ rstd_out, NormArgs na, long long table_rows, int* dbg) {
  const int lane = threadIdx.x % 32;
  const long long row = (long long)blockIdx.x * kWarps + threadIdx.x / 32;
  if (row >= rows) return;
  if (tokens && !in_vocab(tokens[row], table_rows, dbg, kBoundsGather)) return;
  const float* src = tokens ? x + (size_t)tokens[row] * D : x + (size_t)row * D;
  float v[VPL], n[VPL];
#pragma unroll
  for (int i = 0; i < VPL; ++i) v[i] = src[lane + 32 * i];
  float mean, rstd;
  norm_row<VPL>(v, D, eps, na, n, mean, rstd);
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int c = lane + 32 * i;
    const float y = n[i] * gamma[c] + beta[c];
    if (y32) y32[(size_t)row * D + c] = y;
    if (y16) y16[(size_t)row * D + c] = __float2bfloat16_rn(y);
  }
  if (lane == 0) {
    mean_out[row] = mean;
    rstd_out[row] = rstd;
  }
}

// dx = norm^T(dy), with an optional output row remap: input row r = m*H + h with
// m = b*T + t is written to row (b*H + h)*T + t (the [B,H,T,D] layout the attention
// backward GEMMs read). Output bf16 and/or fp32.
template <int VPL>
__global__ void ln_bwd_kernel(const float* __restrict__ dy, const float* __restrict__ x,
                              const float* __restrict__ mean_in, const float* __restrict__ rstd_in, long long rows,
                              int D, const float* __restrict__ gamma, int remap_T, int remap_H,
                              __nv_bfloat16* __restrict__ dx16, float* __restrict__ dx32, float* __restrict__ part,
                              NormArgs na, const int64_t* __restrict__ tokens, long long table_rows, int* dbg) {
  const int lane = threadIdx.x % 32;
  float gam[VPL], dg[VPL], db[VPL], da[VPL], ds[VPL];
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    gam[i] = gamma[lane + 32 * i];
    dg[i] = db[i] = da[i] = ds[i] = 0.f;
  }
  for (long long row = (long long)blockIdx.x * kWarps + threadIdx.x / 32; row < rows;
       row += (long long)gridDim.x * kWarps) {
    float g[VPL], xr[VPL], n[VPL], dx[VPL];
    const float mean = mean_in[row], rstd = rstd_in[row];
    // with `tokens`, x is the embedding table and row r's input is its row tokens[r]
    const bool ok = tokens == nullptr || in_vocab(tokens[row], table_rows, dbg, kBoundsGather);
    const float* xrow = tokens ? x + (size_t)(ok ? tokens[row] : 0) * D : x + (size_t)row * D;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      g[i] = dy[(size_t)row * D + lane + 32 * i];
      xr[i] = xrow[lane + 32 * i];
    }
    norm_row_saved<VPL>(xr, mean, rstd, na, n);
    norm_backward_row<VPL>(g, xr, n, gam, rstd, D, na, dx, dg, db, da, ds);
    long long orow = row;
    if (remap_T > 0) {
      const long long m = row / remap_H, h = row % remap_H;
      const long long b = m / remap_T, t = m % remap_T;
      orow = (b * remap_H + h) * remap_T + t;
    }
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      if (dx16) dx16[(size_t)orow * D + lane + 32 * i] = __float2bfloat16_rn(dx[i]);
      if (dx32) dx32[(size_t)orow * D + lane + 32 * i] = dx[i];
    }
  }
  block_write_partials<VPL>(dg, db, da, ds, D, na.kind, part);
}

// Forward of the residual merge (burn_dragon_core/src/model/residual_stream.rs:511-535):
//   m = sum_s partial[s]  (split-K / per-head partial products of yn @ E)
//   u = norm(m);  v' = norm(v + u)
// Saves m (fp32) and both norms' statistics for the backward.
template <int VPL>
__global__ void tail_fwd_kernel(const float* __restrict__ partial, int nsplit, long long split_stride,
                                const float* __restrict__ v, long long rows, int D, const float* __restrict__ gamma,
                                const float* __restrict__ beta, float eps, float* __restrict__ m_out,
                                float* __restrict__ vout32, __nv_bfloat16* __restrict__ vout16,
                                float* __restrict__ st, NormArgs na) {
  const int lane = threadIdx.x % 32;
  const long long row = (long long)blockIdx.x * kWarps + threadIdx.x / 32;
  if (row >= rows) return;
  float m[VPL], z[VPL], n[VPL];
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    float s = 0.f;
    for (int k = 0; k < nsplit; ++k) s += partial[k * split_stride + (size_t)row * D + lane + 32 * i];
    m[i] = s;
    if (m_out) m_out[(size_t)row * D + lane + 32 * i] = s;
  }
  float mean1, rstd1, mean2, rstd2;
  norm_row<VPL>(m, D, eps, na, n, mean1, rstd1);
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int c = lane + 32 * i;
    z[i] = v[(size_t)row * D + c] + n[i] * gamma[c] + beta[c];
  }
  norm_row<VPL>(z, D, eps, na, n, mean2, rstd2);
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int c = lane + 32 * i;
    const float y = n[i] * gamma[c] + beta[c];
    vout32[(size_t)row * D + c] = y;
    if (vout16) vout16[(size_t)row * D + c] = __float2bfloat16_rn(y);
  }
  if (lane == 0 && st) {
    st[row * 4 + 0] = mean1;
    st[row * 4 + 1] = rstd1;
    st[row * 4 + 2] = mean2;
    st[row * 4 + 3] = rstd2;
  }
}

// Backward of the residual merge. g = d(v'). Writes dm (bf16, operand of the decoder
// backward GEMMs) and dv_res = d(v) through the residual path (fp32).
template <int VPL>
__global__ void tail_bwd_kernel(const float* __restrict__ g_in, const float* __restrict__ v,
                                const float* __restrict__ m_in, const float* __restrict__ st, long long rows, int D,
                                const float* __restrict__ gamma, const float* __restrict__ beta,
                                __nv_bfloat16* __restrict__ dm16, float* __restrict__ dv_res,
                                float* __restrict__ part, NormArgs na) {
  const int lane = threadIdx.x % 32;
  float gam[VPL], bet[VPL], dg[VPL], db[VPL], da[VPL], ds[VPL];
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    gam[i] = gamma[lane + 32 * i];
    bet[i] = beta[lane + 32 * i];
    dg[i] = db[i] = da[i] = ds[i] = 0.f;
  }
  for (long long row = (long long)blockIdx.x * kWarps + threadIdx.x / 32; row < rows;
       row += (long long)gridDim.x * kWarps) {
    const float mean1 = st[row * 4 + 0], rstd1 = st[row * 4 + 1];
    const float mean2 = st[row * 4 + 2], rstd2 = st[row * 4 + 3];
    float g[VPL], mr[VPL], mh[VPL], z[VPL], zh[VPL], dz[VPL], dm[VPL];
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const size_t o = (size_t)row * D + lane + 32 * i;
      g[i] = g_in[o];
      mr[i] = m_in[o];
    }
    norm_row_saved<VPL>(mr, mean1, rstd1, na, mh);
#pragma unroll
    for (int i = 0; i < VPL; ++i) z[i] = v[(size_t)row * D + lane + 32 * i] + mh[i] * gam[i] + bet[i];
    norm_row_saved<VPL>(z, mean2, rstd2, na, zh);
    norm_backward_row<VPL>(g, z, zh, gam, rstd2, D, na, dz, dg, db, da, ds);
    norm_backward_row<VPL>(dz, mr, mh, gam, rstd1, D, na, dm, dg, db, da, ds);
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const size_t o = (size_t)row * D + lane + 32 * i;
      dm16[o] = __float2bfloat16_rn(dm[i]);
      dv_res[o] = dz[i];
    }
  }
  block_write_partials<VPL>(dg, db, da, ds, D, na.kind, part);
}

// out[i] = base[i] (optional) + sum_k p0[k*s0 + i] + sum_k p1[k*s1 + i].
__global__ void sum_rows_kernel(float* __restrict__ out, const float* __restrict__ base, const float* __restrict__ p0,
                                int n0, long long s0, const float* __restrict__ p1, int n1, long long s1,
                                long long total) {
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    float s = base ? base[i] : 0.f;
    for (int k = 0; k < n0; ++k) s += p0[k * s0 + i];
    for (int k = 0; k < n1; ++k) s += p1[k * s1 + i];
    out[i] = s;
  }
}

// Per row: loss = logsumexp(z) - z[target]; dz = (softmax(z) - onehot) * w * inv_count,
// w the optional loss mask (burn_dragon_core/src/model/dragon/language_head.rs:549-572).
template <int VPL>
__global__ void ce_kernel(const float* __restrict__ logits, const int64_t* __restrict__ target,
                          const float* __restrict__ mask, const float* __restrict__ inv_count, long long rows, int V,
                          float* __restrict__ loss_rows, __nv_bfloat16* __restrict__ dlogits, int* dbg) {
  const int lane = threadIdx.x % 32;
  const long long row = (long long)blockIdx.x * kWarps + threadIdx.x / 32;
  if (row >= rows) return;
  if (lane == 0) in_vocab(target[row], V, dbg, kBoundsTarget);
  float z[VPL];
  float mx = -INFINITY;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    z[i] = logits[(size_t)row * V + lane + 32 * i];
    mx = fmaxf(mx, z[i]);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < VPL; ++i) s += expf(z[i] - mx);
  s = warp_sum(s);
  const float lse = mx + logf(s);
  const int64_t tg = target[row];
  const float w = mask ? mask[row] : 1.0f;
  const float sc = w * inv_count[0];
  float zt = 0.f;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int c = lane + 32 * i;
    if (c == tg) zt = z[i];
    const float pr = expf(z[i] - lse);
    dlogits[(size_t)row * V + c] = __float2bfloat16_rn((pr - (c == tg ? 1.f : 0.f)) * sc);
  }
  zt = warp_sum(zt);
  if (lane == 0) loss_rows[row] = (lse - zt) * w;
}

// G[i,j] = P[i,j]*g^(i-j) (j<i) + P[j,i]*g^(j-i) (j>i), 0 on the diagonal, per (b,h)
// T x T block: dS + dS^T of the strictly-causal score matrix, the left factor of
// dQ = (dS + dS^T) Q (the keys equal the queries).
__global__ void symmetrize_kernel(const float* __restrict__ P, __nv_bfloat16* __restrict__ G, int T, int H,
                                  const float* __restrict__ log2_decay) {
  __shared__ float tile[32][33];
  const int bh = blockIdx.z;
  const float* Pb = P + (size_t)bh * T * T;
  __nv_bfloat16* Gb = G + (size_t)bh * T * T;
  const float l2g = log2_decay ? log2_decay[bh % H] : 0.f;
  const int i0 = blockIdx.y * 32, j0 = blockIdx.x * 32;
  for (int r = threadIdx.y; r < 32; r += blockDim.y) tile[r][threadIdx.x] = Pb[(size_t)(j0 + r) * T + i0 + threadIdx.x];
  __syncthreads();
  for (int r = threadIdx.y; r < 32; r += blockDim.y) {
    const int i = i0 + r, j = j0 + threadIdx.x;
    float val = 0.f;
    if (j < i) {
      val = Pb[(size_t)i * T + j];
      if (log2_decay) val *= exp2f((float)(i - j) * l2g);
    } else if (j > i) {
      val = tile[threadIdx.x][r];
      if (log2_decay) val *= exp2f((float)(j - i) * l2g);
    }
    Gb[(size_t)i * T + j] = __float2bfloat16_rn(val);
  }
}

// AdamW (decoupled weight decay) over a flat fp32 buffer, optional device-side gradient
// scale (clipping coefficient) and a bf16 shadow copy for the GEMMs.
__global__ void adamw_kernel(float* __restrict__ p, const float* __restrict__ g, float* __restrict__ m,
                             float* __restrict__ v, __nv_bfloat16* __restrict__ shadow, long long n, float lr,
                             float b1, float b2, float eps, float wd, float bc1, float bc2,
                             const float* __restrict__ gscale, const float* __restrict__ hyper) {
  const float gs = gscale ? gscale[0] : 1.0f;
  if (hyper) {  // device-resident {lr, bc1, bc2}: lets a captured CUDA graph replay every step
    lr = hyper[0];
    bc1 = hyper[1];
    bc2 = hyper[2];
  }
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    const float gi = g[i] * gs;
    const float mi = b1 * m[i] + (1.f - b1) * gi;
    const float vi = b2 * v[i] + (1.f - b2) * gi * gi;
    m[i] = mi;
    v[i] = vi;
    float pi = p[i] * (1.f - lr * wd);
    pi -= lr * (mi / bc1) / (sqrtf(vi / bc2) + eps);
    p[i] = pi;
    if (shadow) shadow[i] = __float2bfloat16_rn(pi);
  }
}

// Embedding-table gradient: out[v, :] (+)= the sum of g[r, :] over the rows r whose token
// is v, added in increasing r (no atomics, so two runs give bitwise equal gradients).
// Block (v, column slab of 256). Without `seg` the block scans every token (the cheap
// choice for byte-sized vocabularies); with `seg` (offsets of a stable token sort, [V + 1])
// it walks only its own rows `perm[seg[v] .. seg[v + 1])`.
__global__ void __launch_bounds__(256) embed_grad_kernel(const int64_t* __restrict__ tokens,
                                                         const int64_t* __restrict__ perm,
                                                         const int64_t* __restrict__ seg,
                                                         const float* __restrict__ g, long long rows, int D,
                                                         float* __restrict__ out, int accumulate, int V, int* dbg) {
  if (dbg != nullptr && blockIdx.x == 0 && blockIdx.y == 0)
    for (long long r = threadIdx.x; r < rows; r += blockDim.x) in_vocab(tokens[r], V, dbg, kBoundsEmbedGrad);
  __shared__ int idx[256];
  __shared__ int wcount[8];
  const int v = blockIdx.x;
  const int col = blockIdx.y * 256 + threadIdx.x;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  float acc = 0.f;
  if (seg != nullptr) {
    if (col < D)
      for (long long i = seg[v]; i < seg[v + 1]; ++i) acc += g[perm[i] * D + col];
  } else {
    for (long long base = 0; base < rows; base += 256) {
      const long long r = base + threadIdx.x;
      const bool hit = r < rows && tokens[r] == v;
      const unsigned m = __ballot_sync(0xffffffffu, hit);
      if (lane == 0) wcount[warp] = __popc(m);
      __syncthreads();
      int off = 0, total = 0;
#pragma unroll
      for (int w = 0; w < 8; ++w) {
        off += w < warp ? wcount[w] : 0;
        total += wcount[w];
      }
      if (hit) idx[off + __popc(m & ((1u << lane) - 1u))] = (int)(r - base);
      __syncthreads();
      if (col < D)
        for (int i = 0; i < total; ++i) acc += g[(base + idx[i]) * D + col];
      __syncthreads();
    }
  }
  if (col < D) {
    float* o = out + (size_t)v * D + col;
    *o = accumulate ? *o + acc : acc;
  }
}

__global__ void sumsq_kernel(const float* __restrict__ x, long long n, float* __restrict__ out) {
  float s = 0.f;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x)
    s += x[i] * x[i];
  s = warp_sum(s);
  __shared__ float sh[32];
  if (threadIdx.x % 32 == 0) sh[threadIdx.x / 32] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < blockDim.x / 32 ? sh[threadIdx.x] : 0.f;
    t = warp_sum(t);
    if (threadIdx.x == 0) atomicAdd(out, t);
  }
}

// [sumsq] -> [sumsq, norm, min(1, max_norm / (norm + 1e-6))]
__global__ void clip_coef_kernel(float* s, float max_norm) {
  const float norm = sqrtf(s[0]);
  s[1] = norm;
  s[2] = fminf(1.0f, max_norm / (norm + 1e-6f));
}

__global__ void cast_bf16_kernel(const float* __restrict__ x, __nv_bfloat16* __restrict__ y, long long n) {
  // 8 elements per step (32-byte loads, one 16-byte store) when both buffers are
  // 16-byte aligned; the scalar loop covers the tail and unaligned buffers
  const long long tid = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const long long nth = (long long)gridDim.x * blockDim.x;
  long long done = 0;
  if ((reinterpret_cast<uintptr_t>(x) % 16 == 0) && (reinterpret_cast<uintptr_t>(y) % 16 == 0)) {
    const long long n8 = n / 8;
    for (long long i = tid; i < n8; i += nth) {
      const float4 a = reinterpret_cast<const float4*>(x)[2 * i];
      const float4 b = reinterpret_cast<const float4*>(x)[2 * i + 1];
      __nv_bfloat162 h[4] = {__floats2bfloat162_rn(a.x, a.y), __floats2bfloat162_rn(a.z, a.w),
                             __floats2bfloat162_rn(b.x, b.y), __floats2bfloat162_rn(b.z, b.w)};
      reinterpret_cast<uint4*>(y)[i] = *reinterpret_cast<uint4*>(h);
    }
    done = n8 * 8;
  }
  for (long long i = done + tid; i < n; i += nth) y[i] = __float2bfloat16_rn(x[i]);
}

}  // namespace

// ====================================================================== host wrappers
namespace {

cudaStream_t cur_stream(const at::Tensor& t) { return at::cuda::getCurrentCUDAStream(t.get_device()).stream(); }

template <typename F>
void dispatch_vpl(int D, F&& f) {
  TORCH_CHECK(D % 32 == 0, "row width ", D, " must be a multiple of 32");
  switch (D / 32) {
    case 1: f(std::integral_constant<int, 1>{}); break;
    case 2: f(std::integral_constant<int, 2>{}); break;
    case 4: f(std::integral_constant<int, 4>{}); break;
    case 8: f(std::integral_constant<int, 8>{}); break;
    case 16: f(std::integral_constant<int, 16>{}); break;
    case 32: f(std::integral_constant<int, 32>{}); break;
    default: TORCH_CHECK(false, "row width ", D, " must be 32 * {1,2,4,8,16,32}");
  }
}

template <typename T>
T* opt_ptr(const c10::optional<at::Tensor>& t) {
  return t ? reinterpret_cast<T*>(t->data_ptr()) : nullptr;
}

// The dgamma/dbeta block reduction needs kWarps * 2 * D floats of dynamic smem (64 KB at
// D = 1024): opt in above the 48 KB default once per kernel.
template <typename K>
void allow_smem(K kern, size_t bytes) {
  if (bytes > 48 * 1024) C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes));
}

NormArgs norm_args(int64_t kind, const c10::optional<at::Tensor>& alpha, const c10::optional<at::Tensor>& shift) {
  TORCH_CHECK(kind >= 0 && kind <= 3, "norm kind must be 0 (layer), 1 (rms), 2 (dynamic tanh) or 3 (derf)");
  if (kind >= 2) TORCH_CHECK(alpha && alpha->scalar_type() == at::kFloat && alpha->is_cuda(), "this norm kind needs alpha");
  if (kind == 3) TORCH_CHECK(shift && shift->scalar_type() == at::kFloat && shift->is_cuda(), "derf needs shift");
  return NormArgs{(int)kind, kind >= 2 ? alpha->data_ptr<float>() : nullptr,
                  kind == 3 ? shift->data_ptr<float>() : nullptr};
}

int part_blocks(long long rows) {
  const long long need = (rows + kWarps - 1) / kWarps;
  return (int)std::min<long long>(need, 148 * 8);
}

}  // namespace

void ln_fwd(const at::Tensor& x, const c10::optional<at::Tensor>& tokens, int64_t rows, int64_t D,
            const at::Tensor& gamma, const at::Tensor& beta, double eps, const c10::optional<at::Tensor>& y32,
            const c10::optional<at::Tensor>& y16, const at::Tensor& mean, const at::Tensor& rstd, int64_t norm_kind, const c10::optional<at::Tensor>& norm_alpha,
            const c10::optional<at::Tensor>& norm_shift) {
  c10::cuda::CUDAGuard g(x.get_device());
  const NormArgs na = norm_args(norm_kind, norm_alpha, norm_shift);
  TORCH_CHECK(x.is_contiguous() && (!tokens || tokens->is_contiguous()), "ln_fwd: inputs must be contiguous");
  const int blocks = (int)((rows + kWarps - 1) / kWarps);
  dispatch_vpl((int)D, [&](auto vpl) {
    ln_fwd_kernel<decltype(vpl)::value><<<blocks, kWarps * 32, 0, cur_stream(x)>>>(
        x.data_ptr<float>(), tokens ? tokens->data_ptr<int64_t>() : nullptr, rows, (int)D, gamma.data_ptr<float>(),
        beta.data_ptr<float>(), (float)eps, opt_ptr<float>(y32), opt_ptr<__nv_bfloat16>(y16), mean.data_ptr<float>(),
        rstd.data_ptr<float>(), na, tokens ? x.size(0) : 0, tokens ? g_debug_word[x.get_device()] : nullptr);
  });
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Returns the [blocks, 2, D] dgamma/dbeta partials.
at::Tensor ln_bwd(const at::Tensor& dy, const at::Tensor& x, const at::Tensor& mean, const at::Tensor& rstd,
                  int64_t rows, int64_t D, const at::Tensor& gamma, int64_t remap_T, int64_t remap_H,
                  const c10::optional<at::Tensor>& dx16, const c10::optional<at::Tensor>& dx32, int64_t norm_kind, const c10::optional<at::Tensor>& norm_alpha,
            const c10::optional<at::Tensor>& norm_shift, const c10::optional<at::Tensor>& tokens) {
  c10::cuda::CUDAGuard g(x.get_device());
  const NormArgs na = norm_args(norm_kind, norm_alpha, norm_shift);
  const int blocks = part_blocks(rows);
  const int R = norm_part_rows(na.kind);
  auto part = at::empty({blocks, R, D}, x.options().dtype(at::kFloat));
  dispatch_vpl((int)D, [&](auto vpl) {
    allow_smem(ln_bwd_kernel<decltype(vpl)::value>, kWarps * R * D * sizeof(float));
    ln_bwd_kernel<decltype(vpl)::value><<<blocks, kWarps * 32, kWarps * R * D * sizeof(float), cur_stream(x)>>>(
        dy.data_ptr<float>(), x.data_ptr<float>(), mean.data_ptr<float>(), rstd.data_ptr<float>(), rows, (int)D,
        gamma.data_ptr<float>(), (int)remap_T, (int)remap_H, opt_ptr<__nv_bfloat16>(dx16), opt_ptr<float>(dx32),
        part.data_ptr<float>(), na, tokens ? tokens->data_ptr<int64_t>() : nullptr, tokens ? x.size(0) : 0,
        tokens ? g_debug_word[x.get_device()] : nullptr);
  });
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return part;
}

void tail_fwd(const at::Tensor& partial, int64_t nsplit, int64_t split_stride, const at::Tensor& v, int64_t rows,
              int64_t D, const at::Tensor& gamma, const at::Tensor& beta, double eps,
              const c10::optional<at::Tensor>& m_out, const at::Tensor& vout32,
              const c10::optional<at::Tensor>& vout16, const c10::optional<at::Tensor>& st, int64_t norm_kind, const c10::optional<at::Tensor>& norm_alpha,
            const c10::optional<at::Tensor>& norm_shift) {
  c10::cuda::CUDAGuard g(v.get_device());
  const NormArgs na = norm_args(norm_kind, norm_alpha, norm_shift);
  const int blocks = (int)((rows + kWarps - 1) / kWarps);
  dispatch_vpl((int)D, [&](auto vpl) {
    tail_fwd_kernel<decltype(vpl)::value><<<blocks, kWarps * 32, 0, cur_stream(v)>>>(
        partial.data_ptr<float>(), (int)nsplit, split_stride, v.data_ptr<float>(), rows, (int)D,
        gamma.data_ptr<float>(), beta.data_ptr<float>(), (float)eps, opt_ptr<float>(m_out), vout32.data_ptr<float>(),
        opt_ptr<__nv_bfloat16>(vout16), opt_ptr<float>(st), na);
  });
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

at::Tensor tail_bwd(const at::Tensor& gin, const at::Tensor& v, const at::Tensor& m, const at::Tensor& st,
                    int64_t rows, int64_t D, const at::Tensor& gamma, const at::Tensor& beta, const at::Tensor& dm16,
                    const at::Tensor& dv_res, int64_t norm_kind, const c10::optional<at::Tensor>& norm_alpha,
            const c10::optional<at::Tensor>& norm_shift) {
  c10::cuda::CUDAGuard g(v.get_device());
  const NormArgs na = norm_args(norm_kind, norm_alpha, norm_shift);
  const int blocks = part_blocks(rows);
  const int R = norm_part_rows(na.kind);
  auto part = at::empty({blocks, R, D}, v.options().dtype(at::kFloat));
  dispatch_vpl((int)D, [&](auto vpl) {
    allow_smem(tail_bwd_kernel<decltype(vpl)::value>, kWarps * R * D * sizeof(float));
    tail_bwd_kernel<decltype(vpl)::value><<<blocks, kWarps * 32, kWarps * R * D * sizeof(float), cur_stream(v)>>>(
        gin.data_ptr<float>(), v.data_ptr<float>(), m.data_ptr<float>(), st.data_ptr<float>(), rows, (int)D,
        gamma.data_ptr<float>(), beta.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(dm16.data_ptr()),
        dv_res.data_ptr<float>(), part.data_ptr<float>(), na);
  });
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return part;
}

void sum_rows(const at::Tensor& out, const c10::optional<at::Tensor>& base, const at::Tensor& p0, int64_t n0,
              int64_t s0, const c10::optional<at::Tensor>& p1, int64_t n1, int64_t s1, int64_t total) {
  c10::cuda::CUDAGuard g(out.get_device());
  sum_rows_kernel<<<148 * 4, 256, 0, cur_stream(out)>>>(out.data_ptr<float>(), opt_ptr<const float>(base),
                                                        p0.data_ptr<float>(), (int)n0, s0, opt_ptr<const float>(p1),
                                                        (int)n1, s1, total);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void cross_entropy(const at::Tensor& logits, const at::Tensor& target, const c10::optional<at::Tensor>& mask,
                   const at::Tensor& inv_count, int64_t rows, int64_t V, const at::Tensor& loss_rows,
                   const at::Tensor& dlogits) {
  c10::cuda::CUDAGuard g(logits.get_device());
  TORCH_CHECK(logits.is_contiguous() && target.is_contiguous(), "cross_entropy: inputs must be contiguous");
  const int blocks = (int)((rows + kWarps - 1) / kWarps);
  dispatch_vpl((int)V, [&](auto vpl) {
    ce_kernel<decltype(vpl)::value><<<blocks, kWarps * 32, 0, cur_stream(logits)>>>(
        logits.data_ptr<float>(), target.data_ptr<int64_t>(), opt_ptr<const float>(mask), inv_count.data_ptr<float>(),
        rows, (int)V, loss_rows.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(dlogits.data_ptr()),
        g_debug_word[logits.get_device()]);
  });
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void symmetrize(const at::Tensor& P, const at::Tensor& G, int64_t BH, int64_t T, int64_t H,
                const c10::optional<at::Tensor>& log2_decay) {
  c10::cuda::CUDAGuard g(P.get_device());
  TORCH_CHECK(T % 32 == 0, "symmetrize needs T % 32 == 0");
  dim3 grid((unsigned)(T / 32), (unsigned)(T / 32), (unsigned)BH);
  symmetrize_kernel<<<grid, dim3(32, 8), 0, cur_stream(P)>>>(
      P.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(G.data_ptr()), (int)T, (int)H,
      opt_ptr<const float>(log2_decay));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void adamw(const at::Tensor& p, const at::Tensor& g, const at::Tensor& m, const at::Tensor& v,
           const c10::optional<at::Tensor>& shadow, double lr, double b1, double b2, double eps, double wd,
           double bc1, double bc2, const c10::optional<at::Tensor>& gscale,
           const c10::optional<at::Tensor>& hyper) {
  c10::cuda::CUDAGuard gd(p.get_device());
  adamw_kernel<<<148 * 8, 256, 0, cur_stream(p)>>>(p.data_ptr<float>(), g.data_ptr<float>(), m.data_ptr<float>(),
                                                   v.data_ptr<float>(), opt_ptr<__nv_bfloat16>(shadow), p.numel(),
                                                   (float)lr, (float)b1, (float)b2, (float)eps, (float)wd,
                                                   (float)bc1, (float)bc2, opt_ptr<const float>(gscale), opt_ptr<const float>(hyper));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Writes [sumsq, norm, clip_coef] into `scratch3` (3 floats).
void grad_clip_coef(const at::Tensor& g, const at::Tensor& scratch3, double max_norm) {
  c10::cuda::CUDAGuard gd(g.get_device());
  C10_CUDA_CHECK(cudaMemsetAsync(scratch3.data_ptr(), 0, sizeof(float), cur_stream(g)));
  sumsq_kernel<<<148 * 4, 256, 0, cur_stream(g)>>>(g.data_ptr<float>(), g.numel(), scratch3.data_ptr<float>());
  clip_coef_kernel<<<1, 1, 0, cur_stream(g)>>>(scratch3.data_ptr<float>(), (float)max_norm);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void embed_grad(const at::Tensor& tokens, const at::Tensor& g, int64_t rows, int64_t D, const at::Tensor& out,
                bool accumulate, const c10::optional<at::Tensor>& perm, const c10::optional<at::Tensor>& seg) {
  c10::cuda::CUDAGuard gd(g.get_device());
  TORCH_CHECK(tokens.is_contiguous() && g.is_contiguous() && out.is_contiguous(), "embed_grad: contiguous inputs");
  TORCH_CHECK(tokens.scalar_type() == at::kLong && g.scalar_type() == at::kFloat && out.scalar_type() == at::kFloat,
              "embed_grad: int64 tokens, fp32 gradient rows and table");
  TORCH_CHECK(tokens.numel() >= rows && g.numel() >= rows * D && out.size(1) == D, "embed_grad: shapes");
  TORCH_CHECK(!perm == !seg, "embed_grad: perm and seg go together");
  const int64_t V = out.size(0);
  if (seg) TORCH_CHECK(seg->numel() == V + 1 && perm->numel() >= rows, "embed_grad: seg needs V + 1 offsets");
  dim3 grid((unsigned)V, (unsigned)((D + 255) / 256));
  embed_grad_kernel<<<grid, 256, 0, cur_stream(g)>>>(tokens.data_ptr<int64_t>(), opt_ptr<const int64_t>(perm),
                                                     opt_ptr<const int64_t>(seg), g.data_ptr<float>(), rows, (int)D,
                                                     out.data_ptr<float>(), accumulate ? 1 : 0, (int)V,
                                                     g_debug_word[g.get_device()]);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Register (or with None clear) the int32 word the bounds checks of `device` report into.
void set_debug_bounds(int64_t device, const c10::optional<at::Tensor>& word) {
  TORCH_CHECK(device >= 0 && device < 64, "device index");
  if (word) TORCH_CHECK(word->scalar_type() == at::kInt && word->is_cuda() && word->get_device() == device,
                        "debug word: an int32 tensor on that device");
  g_debug_word[device] = word ? word->data_ptr<int>() : nullptr;
}

void cast_bf16(const at::Tensor& x, const at::Tensor& y) {
  c10::cuda::CUDAGuard gd(x.get_device());
  cast_bf16_kernel<<<148 * 8, 256, 0, cur_stream(x)>>>(x.data_ptr<float>(),
                                                       reinterpret_cast<__nv_bfloat16*>(y.data_ptr()), x.numel());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace bd
