// gemm_sm100.cuh — the one tensor-core engine every BDH contraction runs on.
//
// A persistent, warp-specialised tcgen05 GEMM for sm_100a:
//   warp 0        : TMA producer (one elected lane) filling a STAGES-deep smem ring
//   warp 1        : TMEM allocator + single-thread tcgen05.mma issuer
//   warps 2..9    : epilogue (two warps per TMEM lane quadrant, each owning half of the
//                   tile's columns), reading fp32 accumulators with tcgen05.ld and
//                   applying a fused, mode-specific epilogue before the global store.
// Two TMEM accumulators (2*BN columns) let the epilogue of tile i overlap the mainloop
// of tile i+1. Tile M is 128, K-block 64 (one 128-byte swizzle atom of bf16), tile N is
// a template parameter (64/128/256). A and B may each be K-major or MN-major in global
// memory; TMA writes them into the canonical 128B-swizzled layouts that the smem
// descriptors describe, so no operand is ever transposed in HBM.
//
// Batching: two batch coordinates (z1, z2) index the 4-D tensor maps of A and B (each
// operand can ignore either coordinate, e.g. the value matrix V shared by all heads)
// and the outputs through element strides. Split-K writes fp32 partials at
// `split * split_stride`; the consumer reduces them.
//
// The reference computes these contractions as scalar FP32 CubeCL/WGSL kernels
// (burn_dragon_kernel/src/relu_lowrank.wgsl:40-82, dense_causal_attention.wgsl:53-106)
// or Burn library matmuls (burn_dragon_core/src/model/dragon/residual_stream.rs:309-321).
#pragma once
#include <cuda_fp16.h>

#include "sm100_ptx.cuh"

namespace bd {

enum EpiMode : int {
  EPI_BF16 = 0,       // out0 = alpha*acc (bf16)
  EPI_F32 = 1,        // out0 (+)= alpha*acc (fp32); split-K partials; out1: bf16 copy of out0
  EPI_RELU_ROPE = 2,  // x = relu(acc - thr) -> out0; q = rope(x, pos) -> out1
  EPI_SCORES = 3,     // strictly-causal masked (and decayed) scores -> out0 (bf16)
  EPI_GATE = 4,       // yn = relu(acc - thr) * x(aux0) -> out0 (bf16)
  EPI_DEC_BWD = 5,    // acc = d(yn): dx_part -> out0, dy_pre -> out1 (aux0 = x, aux1 = yn);
                      // dx_part carries the x <= 0 mask as -0.0
  EPI_DQ = 6,         // acc = d(q): dx_pre = (aux0 + rope^T(acc)), masked by aux0's -0.0 -> out0
  EPI_F32_SCATTER = 7,  // fp32 rows stored straight into their owner rank's slot over NVLink
                        // (the reduce-scatter half of a tensor-parallel sum, fused into the GEMM)
};

struct EpiParams {
  void* out0;
  void* out1;
  const __nv_bfloat16* aux0;
  const __nv_bfloat16* aux1;
  long long ld;            // row stride of outputs/aux (elements)
  long long sz1, sz2;      // batch strides of outputs/aux (elements)
  long long split_stride;  // split-K partial stride (elements)
  float alpha;
  float thr;
  const float* freq;       // RoPE frequency per latent column (cycles / position), or null
  const uint32_t* rope_tab;  // or null: (cos, sin) as half2 per (row % T, column pair), row
                             // stride Nh / 2, phases of positions pos0 + (row % T)
  int rope_tma;            // EPI_RELU_ROPE: the phases come as a staged table (the half2
                           // [T, Nh/2] table of positions pos0 + t, TMA map tx0), not rope_tab
  const float* log2_decay; // per-z1 log2(gamma) for decayed scores, or null
  int T;                   // rows per sequence (position = pos0 + row % T)
  int pos0;
  int Nh;                  // latent per head (column -> in-head index for RoPE)
  int accumulate;          // EPI_F32: add into the existing output
  int row_decay;           // EPI_F32 / EPI_DQ: scale row r by 2^(r * log2_decay[z1])
  const float* acc_src;    // EPI_F32 with accumulate: add this fp32 tensor (same layout as out0)
                           // instead of out0's old contents (out0 = alpha*acc + src*src_scale)
  int src_decay_T;         // > 0: src_scale = 2^(src_decay_T * log2_decay[z1]) (state decay)
  int probe;               // measurement only (BDH_GEMM_PROBE): 1 = TMA-epilogue modes read the
                           // accumulator and release it, skipping aux loads, math and stores
  // EPI_F32_SCATTER: row r belongs to rank r / scatter_rows; it is stored at
  // peer[owner] + scatter_rank * slot_stride + (r % scatter_rows) * ld + col, where
  // peer[] are the (IPC-mapped) slot buffers of every rank. Plain st.global over NVLink.
  float* peer[8];
  int scatter_rows;
  int scatter_rank;
  long long slot_stride;
};

struct alignas(64) GemmParams {
  CUtensorMap ta;
  CUtensorMap tb;
  // TMA-epilogue modes: 32 x 64 boxes (128B swizzle) of the auxiliary inputs / outputs,
  // as 4-D maps (cols, rows, z1, z2) of the output geometry.
  CUtensorMap tx0, tx1, to0, to1;
  int M, N, K;
  int Z1, Z2;
  int tiles_m, tiles_n, splits, kb_per_split;
  int a_z1, a_z2, b_z1, b_z2;  // does the operand's tensor map use z1 / z2?
  int causal_skip;             // tiles with n0 >= m0 + 128 are zero tiles (no MMA)
  int* err;
  EpiParams e;
};

// Epilogue kinds: 0 = fp32 row stores, 1 = register-computed bf16 tiles staged through
// smem (two 4 KB tiles per epilogue warp), 2 = TMA epilogue (aux operands prefetched by
// TMA one tile ahead into double-buffered smem, results stored by TMA; BN = 128 only).
template <int EPI>
constexpr int epi_kind() {
  // 0: fp32 row stores; 1: staged bf16; 2: TMA epilogue, 8 warps x 64 columns, two
  // tile buffers of two tensors; 3: TMA epilogue, 16 warps x 32 columns (the store-only
  // x-projection, where more concurrent warps beat wider boxes); 4: TMA epilogue,
  // 8 warps x 64 columns, a ring of three single-tensor buffers (the gate and dQ: a
  // buffer's store has two tiles to drain before the buffer is refilled)
  return (EPI == EPI_F32 || EPI == EPI_F32_SCATTER) ? 0
         : EPI == EPI_RELU_ROPE                  ? 3
         : (EPI == EPI_GATE || EPI == EPI_DQ)    ? 4
         : EPI == EPI_DEC_BWD                    ? 2
                                                 : 1;
}

// Epilogue warps of the TMA kinds: 16 (four per TMEM lane quadrant, 32-column chunks)
// for the x-projection, else 8 (64-column chunks). (16 warps on 256-wide tiles measured
// slower at BDH-GPU batch 32: twice the TMA operations of half the size.)
constexpr int tma_nepi(int KIND, int BN) { return (KIND == 3 || (KIND >= 2 && BN == 256)) ? 16 : 8; }

template <int BN, int KIND = 0>
struct GemmCfg {
  static constexpr bool STAGED = KIND != 0;
  static constexpr int BM = 128;
  static constexpr int BK = 64;
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = KIND == 4 ? 4 : KIND >= 2 ? 3
                               : (STAGED ? ((BN == 256) ? 3 : (BN == 128 ? 4 : 5))
                                         : ((BN == 256) ? 4 : (BN == 128 ? 6 : 8)));
  // epilogue warps: kind 3 runs 16 (four per TMEM lane quadrant, 32 columns each),
  // the others 8 (two per quadrant, 64 columns each)
  static constexpr int NEPI = KIND >= 2 ? tma_nepi(KIND, BN) : 8;
  // kinds 2 / 3: warps x 2 tile buffers x 2 tensors x (32 rows x columns-per-warp bf16)
  static constexpr int EPI_BYTES = KIND == 4 ? 96 * 1024 : KIND >= 2 ? 128 * 1024 : (STAGED ? 8 * 2 * 4096 : 0);
  static constexpr int SMEM = STAGES * STAGE_BYTES + EPI_BYTES + 1024;
  static constexpr int TMEM_COLS = 2 * BN;
  static constexpr int THREADS = 64 + 32 * NEPI;
};

struct TileCoord {
  int z1, z2, split, m0, n0, kb0, kb1;
  bool zero;
};

__device__ __forceinline__ TileCoord decode_tile(const GemmParams& p, int t, int BN) {
  TileCoord c;
  int n_blk = t % p.tiles_n;
  int r = t / p.tiles_n;
  int m_blk = r % p.tiles_m;
  r /= p.tiles_m;
  c.split = r % p.splits;
  r /= p.splits;
  c.z1 = r % p.Z1;
  c.z2 = r / p.Z1;
  c.m0 = m_blk * 128;
  c.n0 = n_blk * BN;
  const int KB = (p.K + 63) / 64;
  c.kb0 = c.split * p.kb_per_split;
  c.kb1 = min(c.kb0 + p.kb_per_split, KB);
  c.zero = (p.causal_skip && c.n0 >= c.m0 + 128) || (c.kb1 <= c.kb0);
  return c;
}

__device__ __forceinline__ void store_bf16x32(__nv_bfloat16* dst, const float (&v)[32]) {
  uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    __nv_bfloat162 h[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(v[q * 8 + 2 * i], v[q * 8 + 2 * i + 1]);
    d[q] = *reinterpret_cast<uint4*>(h);
  }
}

__device__ __forceinline__ void load_bf16x32(const __nv_bfloat16* src, float (&v)[32]) {
  const uint4* s = reinterpret_cast<const uint4*>(src);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint4 u = s[q];
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 f = __bfloat1622float2(h[i]);
      v[q * 8 + 2 * i] = f.x;
      v[q * 8 + 2 * i + 1] = f.y;
    }
  }
}

// cos/sin of the RoPE phase 2*pi*frac(pos*freq) (phase wrapped as in
// burn_dragon_core/src/model/attention.rs:540-550), evaluated with CUDA's __sincosf on
// the argument reduced to [-pi, pi]: raw - rint(raw) is the phase in revolutions, already
// centred (one rounding instruction in place of floor, compare and subtract).
__device__ __forceinline__ void rope_cs(float pos, float freq, float& c, float& s) {
  const float raw = pos * freq;
  const float ph = (raw - rintf(raw)) * 6.283185307179586f;
  __sincosf(ph, &s, &c);
}

// Apply the epilogue for one thread's 32 consecutive columns of one output row.
// `row`, `col` are coordinates inside the (z1, z2) batch matrix.
template <int EPI>
__device__ __forceinline__ void epilogue_chunk(const GemmParams& p, const TileCoord& tc,
                                               float (&v)[32], int row, int col) {
  const EpiParams& e = p.e;
  if (row >= p.M || col >= p.N) return;
  const long long off = (long long)tc.z2 * e.sz2 + (long long)tc.z1 * e.sz1 + (long long)row * e.ld + col;
  if constexpr (EPI == EPI_F32_SCATTER) {
    const int owner = row / e.scatter_rows;
    float4* o4 = reinterpret_cast<float4*>(e.peer[owner] + (long long)e.scatter_rank * e.slot_stride +
                                           (long long)(row - owner * e.scatter_rows) * e.ld + col);
#pragma unroll
    for (int q = 0; q < 8; ++q) o4[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
    return;
  } else if constexpr (EPI == EPI_F32) {
    float* o = reinterpret_cast<float*>(e.out0) + off + (long long)tc.split * e.split_stride;
    float4* o4 = reinterpret_cast<float4*>(o);
    const float a = e.row_decay ? e.alpha * exp2f((float)row * e.log2_decay[tc.z1]) : e.alpha;
    // out1 (optional): a bf16 copy of the stored fp32 values (the state GEMM's next-chunk
    // operand), so no separate conversion pass reads the fp32 result back
    __nv_bfloat162* o16 = e.out1 ? reinterpret_cast<__nv_bfloat162*>(reinterpret_cast<__nv_bfloat16*>(e.out1) + off +
                                                                     (long long)tc.split * e.split_stride)
                                 : nullptr;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      float4 w = make_float4(a * v[4 * q], a * v[4 * q + 1], a * v[4 * q + 2], a * v[4 * q + 3]);
      if (e.accumulate) {
        float4 old = e.acc_src ? reinterpret_cast<const float4*>(e.acc_src + off)[q] : o4[q];
        if (e.src_decay_T > 0) {
          const float sc = exp2f((float)e.src_decay_T * e.log2_decay[tc.z1]);
          old.x *= sc; old.y *= sc; old.z *= sc; old.w *= sc;
        }
        w.x += old.x; w.y += old.y; w.z += old.z; w.w += old.w;
      }
      o4[q] = w;
      if (o16) {
        o16[2 * q] = __floats2bfloat162_rn(w.x, w.y);
        o16[2 * q + 1] = __floats2bfloat162_rn(w.z, w.w);
      }
    }
    return;
  } else {
    if constexpr (EPI == EPI_BF16) {
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] *= e.alpha;
    } else if constexpr (EPI == EPI_RELU_ROPE) {
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = fmaxf(v[i] - e.thr, 0.0f);
    } else if constexpr (EPI == EPI_SCORES) {
      const float l2g = e.log2_decay ? e.log2_decay[tc.z1] : 0.0f;
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const int c = col + i;
        float w = (c < row) ? v[i] : 0.0f;
        if (e.log2_decay && c < row) w *= exp2f((float)(row - c) * l2g);
        v[i] = w;
      }
    } else if constexpr (EPI == EPI_GATE) {
      float xv[32];
      load_bf16x32(e.aux0 + off, xv);
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = fmaxf(v[i] - e.thr, 0.0f) * xv[i];
    }
    __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(e.out0) + off;
    store_bf16x32(o, v);
    if constexpr (EPI == EPI_RELU_ROPE) {
      if (e.freq) {
        const float pos = (float)(e.pos0 + row % e.T);
        const int j0 = col % e.Nh;
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          float c, s;
          rope_cs(pos, e.freq[j0 + i], c, s);
          const float xe = v[i], xo = v[i + 1];
          v[i] = xe * c - xo * s;
          v[i + 1] = xo * c + xe * s;
        }
        store_bf16x32(reinterpret_cast<__nv_bfloat16*>(e.out1) + off, v);
      }
    }
  }
}

template <int EPI>
__device__ __forceinline__ void epilogue_zero_chunk(const GemmParams& p, const TileCoord& tc,
                                                    int row, int col) {
  float v[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = 0.0f;
  if (row >= p.M || col >= p.N) return;
  const EpiParams& e = p.e;
  const long long off = (long long)tc.z2 * e.sz2 + (long long)tc.z1 * e.sz1 + (long long)row * e.ld + col;
  if constexpr (EPI == EPI_F32_SCATTER) {
    return;  // the scattered GEMM has no zero tiles (no causal skip, K > 0)
  } else if constexpr (EPI == EPI_F32) {
    if (e.accumulate) return;  // (a zero tile leaves an accumulated output, and its copy, as it is)
    float4* o4 = reinterpret_cast<float4*>(reinterpret_cast<float*>(e.out0) + off +
                                           (long long)tc.split * e.split_stride);
#pragma unroll
    for (int q = 0; q < 8; ++q) o4[q] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (e.out1) {
      uint4* o16 = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(e.out1) + off +
                                            (long long)tc.split * e.split_stride);
#pragma unroll
      for (int q = 0; q < 4; ++q) o16[q] = make_uint4(0u, 0u, 0u, 0u);
    }
  } else {
    store_bf16x32(reinterpret_cast<__nv_bfloat16*>(e.out0) + off, v);
  }
}

}  // namespace bd

namespace bd {

// Tile of a CTA pair: rows [m0, m0 + 256); the caller adds 128 * cta_rank.
__device__ __forceinline__ TileCoord decode_tile_pair(const GemmParams& p, int t, int BN) {
  TileCoord c;
  int n_blk = t % p.tiles_n;
  int r = t / p.tiles_n;
  int m_blk = r % p.tiles_m;
  r /= p.tiles_m;
  c.split = r % p.splits;
  r /= p.splits;
  c.z1 = r % p.Z1;
  c.z2 = r / p.Z1;
  c.m0 = m_blk * 256;
  c.n0 = n_blk * BN;
  const int KB = (p.K + 63) / 64;
  c.kb0 = c.split * p.kb_per_split;
  c.kb1 = min(c.kb0 + p.kb_per_split, KB);
  c.zero = (p.causal_skip && c.n0 >= c.m0 + 256) || (c.kb1 <= c.kb0);
  return c;
}

}  // namespace bd

#include "gemm_epilogue_staged.cuh"
#include "gemm_epilogue_tma.cuh"
#include "gemm_sm100_kernel.cuh"
