// gemm_epilogue_staged.cuh — coalesced epilogue for the bf16-output modes.
//
// After tcgen05.ld each thread owns one output row. Storing (or loading auxiliary
// operands) row-per-thread makes every warp-wide 16-byte access touch 32 different
// cache lines. Instead each epilogue warp stages its 32 x 64 chunk in two private
// 4 KB shared-memory tiles: rows of 128 bytes whose 16-byte chunk index is XOR-ed with
// (row & 7), so both the row-per-thread accesses and the line-per-4-lanes accesses are
// bank-conflict free; global traffic then moves whole 128-byte rows, 4 rows per warp
// instruction.
#pragma once

namespace bd {

constexpr int kStageTileBytes = 32 * 128;  // one 32 x 64 bf16 tile

__device__ __forceinline__ uint32_t stg_off(int row, int chunk) {
  return (uint32_t)(row * 128 + ((chunk ^ (row & 7)) << 4));
}

__device__ __forceinline__ uint4 pack8(const float* w) {
  __nv_bfloat162 h[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(w[2 * i], w[2 * i + 1]);
  return *reinterpret_cast<uint4*>(h);
}

__device__ __forceinline__ void unpack8(uint4 u, float* w) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 f = __bfloat1622float2(h[i]);
    w[2 * i] = f.x;
    w[2 * i + 1] = f.y;
  }
}

// Global [32 x 64] tile at g (row stride ld) -> staging buffer, zero outside the valid box.
__device__ __forceinline__ void coop_load(const __nv_bfloat16* g, long long ld, int rows_valid, int cols_valid,
                                          uint8_t* buf, int lane) {
  uint4 r[8];
  const int ch = lane & 7;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const int row = 4 * k + (lane >> 3);
    const bool ok = row < rows_valid && ch * 8 < cols_valid;
    r[k] = ok ? *reinterpret_cast<const uint4*>(g + row * ld + ch * 8) : make_uint4(0u, 0u, 0u, 0u);
  }
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const int row = 4 * k + (lane >> 3);
    *reinterpret_cast<uint4*>(buf + stg_off(row, ch)) = r[k];
  }
}

__device__ __forceinline__ void coop_store(__nv_bfloat16* g, long long ld, int rows_valid, int cols_valid,
                                           const uint8_t* buf, int lane) {
  const int ch = lane & 7;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const int row = 4 * k + (lane >> 3);
    if (row < rows_valid && ch * 8 < cols_valid)
      *reinterpret_cast<uint4*>(g + row * ld + ch * 8) = *reinterpret_cast<const uint4*>(buf + stg_off(row, ch));
  }
}

__device__ __forceinline__ void coop_zero(__nv_bfloat16* g, long long ld, int rows_valid, int cols_valid, int lane) {
  const int ch = lane & 7;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const int row = 4 * k + (lane >> 3);
    if (row < rows_valid && ch * 8 < cols_valid)
      *reinterpret_cast<uint4*>(g + row * ld + ch * 8) = make_uint4(0u, 0u, 0u, 0u);
  }
}

// One warp, 32 rows (row_base .. row_base+31 of the batch matrix) x 64 columns.
template <int EPI>
__device__ __forceinline__ void epilogue_chunk64(const GemmParams& p, const TileCoord& tc, float (&v)[64],
                                                 int row_base, int col0, uint8_t* buf0, uint8_t* buf1,
                                                 int lane) {
  const EpiParams& e = p.e;
  const int rows_valid = min(32, p.M - row_base);
  if (rows_valid <= 0 || col0 >= p.N) return;
  const int cols_valid = min(64, p.N - col0);
  const long long base = (long long)tc.z2 * e.sz2 + (long long)tc.z1 * e.sz1 + (long long)row_base * e.ld + col0;
  const int row = row_base + lane;

  if constexpr (EPI == EPI_GATE) {
    coop_load(e.aux0 + base, e.ld, rows_valid, cols_valid, buf0, lane);
  }
  static_assert(EPI != EPI_DEC_BWD && EPI != EPI_DQ, "decoder-backward and dQ use the TMA epilogue");
  __syncwarp();

  float pos = 0.f;
  int j0 = 0;
  if constexpr (EPI == EPI_RELU_ROPE) {
    pos = (float)(e.pos0 + row % e.T);
    j0 = col0 % e.Nh;
  }
  float l2g = 0.f;
  if constexpr (EPI == EPI_SCORES) {
    if (e.log2_decay) l2g = e.log2_decay[tc.z1];
  }

#pragma unroll
  for (int c = 0; c < 8; ++c) {
    float* w = v + 8 * c;
    if constexpr (EPI == EPI_BF16) {
#pragma unroll
      for (int i = 0; i < 8; ++i) w[i] *= e.alpha;
      *reinterpret_cast<uint4*>(buf0 + stg_off(lane, c)) = pack8(w);
    } else if constexpr (EPI == EPI_SCORES) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int col = col0 + 8 * c + i;
        float s = (col < row) ? w[i] : 0.0f;
        if (e.log2_decay && col < row) s *= exp2f((float)(row - col) * l2g);
        w[i] = s;
      }
      *reinterpret_cast<uint4*>(buf0 + stg_off(lane, c)) = pack8(w);
    } else if constexpr (EPI == EPI_RELU_ROPE) {
#pragma unroll
      for (int i = 0; i < 8; ++i) w[i] = fmaxf(w[i] - e.thr, 0.0f);
      *reinterpret_cast<uint4*>(buf0 + stg_off(lane, c)) = pack8(w);
      if (e.freq) {
        const float4 fa = *reinterpret_cast<const float4*>(e.freq + j0 + 8 * c);
        const float4 fb = *reinterpret_cast<const float4*>(e.freq + j0 + 8 * c + 4);
        const float f[4] = {fa.x, fa.z, fb.x, fb.z};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          float cs, sn;
          rope_cs(pos, f[i], cs, sn);
          const float xe = w[2 * i], xo = w[2 * i + 1];
          w[2 * i] = xe * cs - xo * sn;
          w[2 * i + 1] = xo * cs + xe * sn;
        }
        *reinterpret_cast<uint4*>(buf1 + stg_off(lane, c)) = pack8(w);
      }
    } else if constexpr (EPI == EPI_GATE) {
      float xv[8];
      unpack8(*reinterpret_cast<const uint4*>(buf0 + stg_off(lane, c)), xv);
#pragma unroll
      for (int i = 0; i < 8; ++i) w[i] = fmaxf(w[i] - e.thr, 0.0f) * xv[i];
      *reinterpret_cast<uint4*>(buf0 + stg_off(lane, c)) = pack8(w);
    }
  }
  __syncwarp();
  coop_store(reinterpret_cast<__nv_bfloat16*>(e.out0) + base, e.ld, rows_valid, cols_valid, buf0, lane);
  if constexpr (EPI == EPI_DEC_BWD) {
    coop_store(reinterpret_cast<__nv_bfloat16*>(e.out1) + base, e.ld, rows_valid, cols_valid, buf1, lane);
  } else if constexpr (EPI == EPI_RELU_ROPE) {
    if (e.freq)
      coop_store(reinterpret_cast<__nv_bfloat16*>(e.out1) + base, e.ld, rows_valid, cols_valid, buf1, lane);
  }
  __syncwarp();
}

template <int EPI>
__device__ __forceinline__ void epilogue_zero64(const GemmParams& p, const TileCoord& tc, int row_base, int col0,
                                                int lane) {
  const EpiParams& e = p.e;
  const int rows_valid = min(32, p.M - row_base);
  if (rows_valid <= 0 || col0 >= p.N) return;
  const int cols_valid = min(64, p.N - col0);
  const long long base = (long long)tc.z2 * e.sz2 + (long long)tc.z1 * e.sz1 + (long long)row_base * e.ld + col0;
  coop_zero(reinterpret_cast<__nv_bfloat16*>(e.out0) + base, e.ld, rows_valid, cols_valid, lane);
}

}  // namespace bd
