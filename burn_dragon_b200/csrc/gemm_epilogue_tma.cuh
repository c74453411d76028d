// gemm_epilogue_tma.cuh — asynchronous epilogue for the memory-bound BDH modes
// (x-projection + RoPE, gate, decoder backward, dQ), tile N = 128 or 256.
//
// Each epilogue warp owns a 32-row x CW-column chunk of every tile: CW = 64 with 8
// warps (128-byte rows, 128B swizzle) or CW = 32 with 16 warps (64-byte rows, 64B
// swizzle). A warp's auxiliary operands (x, yn, dx_part) are fetched by TMA one tile
// ahead into a double-buffered smem tile pair, so the fetch overlaps the current tile's
// math and store; results are written over the aux tile in place and leave through TMA
// bulk stores. No warp ever waits on a global load of its own, and the accumulator is handed
// back to the MMA warp right after tcgen05.ld, before the math.
#pragma once

namespace bd {

// Byte offset of 16-byte chunk `chunk` (0..3) of row `row` in a 32 x 32 bf16 tile laid
// out by a TMA SWIZZLE_64B box: 64-byte rows, chunk index XOR address bits 7..8.
__device__ __forceinline__ uint32_t sw64_off(int row, int chunk) {
  return (uint32_t)(row * 64 + ((chunk ^ ((row >> 1) & 3)) << 4));
}

template <int EPI>
constexpr int epi_naux() {
  return (EPI == EPI_GATE || EPI == EPI_DQ) ? 1 : (EPI == EPI_DEC_BWD ? 2 : 0);
}

// The x > 0 mask rides in dx_part: the decoder backward writes -0.0 (bf16 0x8000) where
// x <= 0 and never writes -0.0 elsewhere, so no live entry carries the 0x8000 pattern; dQ
// reads the mask from those bits instead of re-reading x, and keeps the marker in its
// output for a second dQ pass over the same buffer.

// In-place math on the smem tiles b0 (and b1) for this thread's row.
template <int CW>
__device__ __forceinline__ uint32_t epi_off(int row, int chunk) {
  if constexpr (CW == 32)
    return sw64_off(row, chunk);
  else
    return stg_off(row, chunk);
}

// cos / sin of the RoPE phases of latent pairs j/2 .. j/2 + 3 at table row `trow` (the
// position pos0 + trow): from the half2 table when the call has one (one 16-byte load for
// four pairs), else evaluated from the frequencies.
__device__ __forceinline__ void rope_cs4(const EpiParams& e, float pos, int trow, int j, float (&cs)[4],
                                         float (&sn)[4]) {
  if (e.rope_tab) {
    const uint4 u = *reinterpret_cast<const uint4*>(e.rope_tab + (size_t)trow * (e.Nh >> 1) + (j >> 1));
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
      cs[i] = f.x;
      sn[i] = f.y;
    }
  } else {
    const float4 fa = *reinterpret_cast<const float4*>(e.freq + j);
    const float4 fb = *reinterpret_cast<const float4*>(e.freq + j + 4);
    const float f[4] = {fa.x, fa.z, fb.x, fb.z};
#pragma unroll
    for (int i = 0; i < 4; ++i) rope_cs(pos, f[i], cs[i], sn[i]);
  }
}

// cos / sin of four consecutive RoPE pairs from one 16-byte word of the staged half2 table.
__device__ __forceinline__ void rope_cs4_word(uint4 u, float (&cs)[4], float (&sn)[4]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
    cs[i] = f.x;
    sn[i] = f.y;
  }
}

template <int EPI, int CW>
__device__ __forceinline__ void tma_epi_math(const GemmParams& p, const TileCoord& tc, float (&v)[CW], int row,
                                             int col0, uint8_t* b0, uint8_t* b1, int lane) {
  const EpiParams& e = p.e;
  float pos = 0.f;
  int j0 = 0, trow = 0;
  if constexpr (EPI == EPI_RELU_ROPE) {
    trow = row % e.T;
    pos = (float)(e.pos0 + trow);
    j0 = col0 % e.Nh;
  } else if constexpr (EPI == EPI_DQ) {
    trow = row;
    pos = (float)(e.pos0 + row);
    j0 = col0;
    if (e.row_decay) {
      const float a = exp2f((float)row * e.log2_decay[tc.z1]);
#pragma unroll
      for (int i = 0; i < CW; ++i) v[i] *= a;
    }
  }
#pragma unroll
  for (int c = 0; c < CW / 8; ++c) {
    float* w = v + 8 * c;
    uint4* s0 = reinterpret_cast<uint4*>(b0 + epi_off<CW>(lane, c));
    uint4* s1 = reinterpret_cast<uint4*>(b1 + epi_off<CW>(lane, c));
    if constexpr (EPI == EPI_RELU_ROPE) {
      // with a staged phase table, its word for these four pairs sits where x goes
      const uint4 tw = e.rope_tma ? *s0 : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
      for (int i = 0; i < 8; ++i) w[i] = fmaxf(w[i] - e.thr, 0.0f);
      *s0 = pack8(w);
      if (e.freq) {
        float cs[4], sn[4];
        if (e.rope_tma)
          rope_cs4_word(tw, cs, sn);
        else
          rope_cs4(e, pos, trow, j0 + 8 * c, cs, sn);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float xe = w[2 * i], xo = w[2 * i + 1];
          w[2 * i] = xe * cs[i] - xo * sn[i];
          w[2 * i + 1] = xo * cs[i] + xe * sn[i];
        }
        *s1 = pack8(w);
      }
    } else if constexpr (EPI == EPI_GATE) {
      float xv[8];
      unpack8(*s0, xv);
#pragma unroll
      for (int i = 0; i < 8; ++i) w[i] = fmaxf(w[i] - e.thr, 0.0f) * xv[i];
      *s0 = pack8(w);
    } else if constexpr (EPI == EPI_DEC_BWD) {
      float xv[8], yv[8], dy[8];
      unpack8(*s0, xv);
      unpack8(*s1, yv);
      // x >= 0 and yn = y x >= 0, so yn > 0 implies x > 0. dx_part = g yn / x on live
      // entries: adding +0.0 turns an exact -0.0 quotient (g < 0, yn = 0) into +0.0, so a
      // live entry never carries the mask pattern (a nonzero quotient keeps its sign and
      // rounds to a nonzero bf16 unless its magnitude is below 1e-40).
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float g = w[i];
        dy[i] = yv[i] > 0.0f ? g * xv[i] : 0.0f;
        const float dxp = __fdividef(g * yv[i], xv[i]) + 0.0f;
        w[i] = xv[i] > 0.0f ? dxp : -0.0f;
      }
      *s0 = pack8(w);
      *s1 = pack8(dy);
    } else if constexpr (EPI == EPI_DQ) {
      float bv[8];
      unpack8(*s0, bv);
      if (e.freq) {
        float cs[4], sn[4];
        rope_cs4(e, pos, trow, j0 + 8 * c, cs, sn);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float ge = w[2 * i], go = w[2 * i + 1];
          w[2 * i] = ge * cs[i] + go * sn[i];
          w[2 * i + 1] = go * cs[i] - ge * sn[i];
        }
      }
      // a masked entry is exactly -0.0 (0x80000000 once widened); a live entry is never
      // -0.0, and w + bv of a live entry is -0.0 only if both are, so the sum needs no flush
#pragma unroll
      for (int i = 0; i < 8; ++i) w[i] = __float_as_uint(bv[i]) == 0x80000000u ? -0.0f : w[i] + bv[i];
      *s0 = pack8(w);
    }
  }
}

// The epilogue warps' loop over this CTA's tiles (tile t0, t0 + tstep, ...). PAIR: the
// tiles are CTA-pair tiles (rows shifted by row_shift for this CTA) and the accumulator
// is released on the leader CTA's tmem-empty barrier.
//
// Warp ew owns TMEM lane quadrant (warp % 4) and column group ew / 4 of width
// GW = BN / (NEPI / 4); it walks its group in chunks of CW columns (CH = GW / CW chunks
// per tile: 1 for BN = 128, 2 for BN = 256). Each chunk is one unit of the per-warp
// buffer ring: the aux tiles of the next unit are fetched while this one is computed.
// The accumulator is handed back after the tile's last chunk has been read from TMEM.
template <int BN, int EPI, int KIND, bool PAIR>
__device__ __forceinline__ void tma_epilogue_loop(const GemmParams& p, int total, int t0, int tstep, int row_shift,
                                                  uint8_t* sEpi, uint64_t (*aux_bar)[3], uint64_t* tfull_bar,
                                                  uint64_t* tempty_bar, uint32_t leader_tempty0,
                                                  uint32_t leader_tempty1, bool leader, uint32_t tmem_base,
                                                  volatile int* abort_flag, int warp, int lane) {
  constexpr int NAUX = epi_naux<EPI>();
  constexpr int NEPI = tma_nepi(KIND, BN);
  constexpr int CW = NEPI == 16 ? 32 : 64;  // columns per chunk
  constexpr int GW = BN / (NEPI / 4);      // columns per warp and tile
  constexpr int CH = GW / CW;              // chunks per warp and tile
  static_assert(CH >= 1 && GW % CW == 0, "tile N must be a multiple of the warp column group");
  constexpr int kTmaTileBytes = 32 * CW * 2;
  constexpr int NBUF = KIND == 4 ? 3 : 2;  // ring of tile buffers
  constexpr int TENS = KIND == 4 ? 1 : 2;  // tensors per buffer
  const int ew = warp - 2;
  const int quad = warp & 3;  // TMEM lane quadrant this warp may access
  const int r_local = quad * 32 + lane;
  uint8_t* wbuf = sEpi + ew * NBUF * TENS * kTmaTileBytes;  // [buffer][tensor] tiles
  const int grp_off = (ew >> 2) * GW;
  auto tile = [&](int t) {
    if constexpr (PAIR) {
      TileCoord c = decode_tile_pair(p, t, BN);
      c.m0 += row_shift;
      return c;
    } else {
      return decode_tile(p, t, BN);
    }
  };
  // Unit u (a chunk of a tile) uses aux buffer u % NBUF for the (u / NBUF)-th time, so its
  // mbarrier parity is (u / NBUF) & 1; `issued_upto` / `waited_upto` (uniform across the
  // warp; only lane 0 issues) bound the loads still landing when the loop ends early.
  int issued_upto = -1, waited_upto = -1;
  // aux fetch of chunk c of tile t into buffer b (no zero tiles in these modes)
  // measurement switches (BDH_GEMM_PROBE bits): 1 = read and release the accumulator
  // only; 2 = store the results with coalesced st.global from the staging tile instead
  // of TMA; 4 = load the aux tiles with coalesced ld.global at use instead of TMA
  // prefetch (2 and 4 apply to the 64-column kinds)
  const bool probe = (p.e.probe & 1) != 0;
  const bool dstore = CW == 64 && (p.e.probe & 2) != 0;
  const bool dload = CW == 64 && (p.e.probe & 4) != 0;
  // The x-projection's RoPE phases may come as a staged table: a [T, Nh/2] half2 (cos, sin)
  // tensor whose 32-row x CW/2-pair box has the byte geometry of a bf16 output box, fetched
  // into the buffer x is then written over.
  const bool tab = EPI == EPI_RELU_ROPE && p.e.rope_tma != 0;
  const bool has_aux = NAUX > 0 || tab;
  auto issue_aux = [&](int t, int c, int u) {
    if (!has_aux) return;
    if (t >= total || probe || dload) return;
    const TileCoord n = tile(t);
    if (n.zero) return;
    issued_upto = u;
    const int b = u % NBUF;
    if (lane != 0) return;
    uint8_t* dst = wbuf + b * TENS * kTmaTileBytes;
    const int col = n.n0 + grp_off + c * CW;
    fence_proxy_async_smem();
    if (tab) {
      mbar_arrive_expect_tx(&aux_bar[ew][b], kTmaTileBytes);
      tma_load_4d(dst, &p.tx0, &aux_bar[ew][b], col >> 1, (n.m0 + quad * 32) % p.e.T, 0, 0);
      return;
    }
    if constexpr (NAUX > 0) {
      mbar_arrive_expect_tx(&aux_bar[ew][b], NAUX * kTmaTileBytes);
      tma_load_4d(dst, &p.tx0, &aux_bar[ew][b], col, n.m0 + quad * 32, n.z1, n.z2);
      if constexpr (NAUX > 1)
        tma_load_4d(dst + kTmaTileBytes, &p.tx1, &aux_bar[ew][b], col, n.m0 + quad * 32, n.z1, n.z2);
    }
  };
  issue_aux(t0, 0, 0);  // unit 0
  int acc = 0;
  uint32_t acc_phase = 0;
  int it = 0;
  bool ok = true;
  for (int t = t0; t < total && ok; t += tstep) {
    const TileCoord tc = tile(t);
    if (tc.zero) continue;  // (no zero tiles in these modes unless K is empty)
#pragma unroll 1
    for (int c = 0; c < CH; ++c, ++it) {
      const int b = it % NBUF;
      uint8_t* b0 = wbuf + b * TENS * kTmaTileBytes;
      uint8_t* b1 = TENS > 1 ? b0 + kTmaTileBytes : b0;
      // the next buffer was last read by this warp's stores NBUF - 1 units ago; with no
      // aux prefetch (x-projection) only this unit's buffer, stored two units ago, must be
      // free, so the previous unit's store may still be reading
      if (lane == 0) {
        if (NBUF == 3 || !has_aux)
          bulk_wait_group_read1();
        else
          bulk_wait_group_read0();
      }
      __syncwarp();
      if (c + 1 < CH)
        issue_aux(t, c + 1, it + 1);
      else
        issue_aux(t + tstep, 0, it + 1);
      if (c == 0) {
        if (!mbar_wait_bounded(&tfull_bar[acc], acc_phase, abort_flag, p.err, kErrTimeoutEpilogue)) {
          ok = false;
          break;
        }
        tc_fence_after();
      }
      const int col_off = grp_off + c * CW;
      float v[CW];
      if constexpr (CW == 32)
        tmem_ld32(tmem_base + ((uint32_t)(quad * 32) << 16) + acc * BN + col_off, v);
      else
        tmem_ld64(tmem_base + ((uint32_t)(quad * 32) << 16) + acc * BN + col_off, v);
      if (c == CH - 1) {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if (!PAIR || leader)
            mbar_arrive(&tempty_bar[acc]);
          else
            mbar_arrive_cluster(acc ? leader_tempty1 : leader_tempty0);
        }
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
      if (probe) {
        // keep the TMEM load live so it is not optimised away
        if (v[0] == 1.2345e-30f && p.e.alpha == -7.0f) *reinterpret_cast<float*>(p.e.out0) = v[1];
        continue;
      }
      const long long goff = (long long)tc.z2 * p.e.sz2 + (long long)tc.z1 * p.e.sz1 +
                             (long long)(tc.m0 + quad * 32) * p.e.ld + tc.n0 + col_off;
      const int rows_ok = min(32, p.M - (tc.m0 + quad * 32)), cols_ok = min(CW, p.N - (tc.n0 + col_off));
      if (has_aux) {
        if (dload && NAUX > 0) {
          coop_load(p.e.aux0 + goff, p.e.ld, rows_ok, cols_ok, b0, lane);
          if constexpr (NAUX > 1) coop_load(p.e.aux1 + goff, p.e.ld, rows_ok, cols_ok, b1, lane);
          __syncwarp();
        } else {
          if (!mbar_wait_bounded(&aux_bar[ew][b], (uint32_t)((it / NBUF) & 1), abort_flag, p.err,
                                 kErrTimeoutEpilogue)) {
            ok = false;
            break;
          }
          waited_upto = it;
        }
      }
      tma_epi_math<EPI, CW>(p, tc, v, tc.m0 + r_local, tc.n0 + col_off, b0, b1, lane);
      if (dstore) {
        __syncwarp();
        coop_store(reinterpret_cast<__nv_bfloat16*>(p.e.out0) + goff, p.e.ld, rows_ok, cols_ok, b0, lane);
        if (EPI == EPI_DEC_BWD)
          coop_store(reinterpret_cast<__nv_bfloat16*>(p.e.out1) + goff, p.e.ld, rows_ok, cols_ok, b1, lane);
        __syncwarp();
        continue;
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        const int c0 = tc.n0 + col_off, c1 = tc.m0 + quad * 32;
        tma_store_4d(&p.to0, b0, c0, c1, tc.z1, tc.z2);
        if (EPI == EPI_DEC_BWD || (EPI == EPI_RELU_ROPE && p.e.freq != nullptr))
          tma_store_4d(&p.to1, b1, c0, c1, tc.z1, tc.z2);
        bulk_commit_group();
      }
    }
  }
  if (lane == 0) {
    bulk_wait_group0();
    // On an abort, loads may still be landing in smem: wait for them (bounded).
    int dummy_abort = 0;
    for (int u = waited_upto + 1; u <= issued_upto; ++u)
      mbar_wait_bounded(&aux_bar[ew][u % NBUF], (uint32_t)((u / NBUF) & 1), (volatile int*)&dummy_abort, p.err,
                        kErrTimeoutDrain);
  }
  __syncwarp();
}

}  // namespace bd
