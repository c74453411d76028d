// gemm_sm100_kernel.cuh — the persistent warp-specialised tcgen05 GEMM kernel body.
// Included from gemm_sm100.cuh (parameter structs and epilogues live there).
#pragma once

namespace bd {

template <int BN, bool A_MN, bool B_MN, int EPI>
__global__ void __launch_bounds__(GemmCfg<BN, epi_kind<EPI>()>::THREADS, 1)
    gemm_sm100_kernel(const __grid_constant__ GemmParams p) {
  constexpr int KIND = epi_kind<EPI>();
  constexpr bool STAGED = KIND == 1;
  static_assert(KIND < 2 || BN == 128 || BN == 256, "the TMA epilogue is built for tile N = 128 / 256");
  using Cfg = GemmCfg<BN, KIND>;
  constexpr int STAGES = Cfg::STAGES;
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint64_t full_bar[STAGES];
  __shared__ uint64_t empty_bar[STAGES];
  __shared__ uint64_t tfull_bar[2];
  __shared__ uint64_t tempty_bar[2];
  __shared__ uint64_t drain_bar;
  __shared__ uint32_t tmem_base_s;
  __shared__ volatile int abort_flag;
  __shared__ uint64_t aux_bar[16][3];

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * Cfg::A_BYTES;
  uint8_t* sEpi = smem + STAGES * Cfg::STAGE_BYTES;

  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], Cfg::NEPI);
    }
    mbar_init(&drain_bar, 1);
    for (int w = 0; w < Cfg::NEPI; ++w) {
      mbar_init(&aux_bar[w][0], 1);
      mbar_init(&aux_bar[w][1], 1);
      mbar_init(&aux_bar[w][2], 1);
    }
    fence_barrier_init();
    tma_prefetch_desc(&p.ta);
    tma_prefetch_desc(&p.tb);
  }
  if (warp == 1) tmem_alloc(&tmem_base_s, Cfg::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = tmem_base_s;

  const int total = p.tiles_m * p.tiles_n * p.splits * p.Z1 * p.Z2;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------ TMA producer
      int stage = 0;
      uint32_t phase = 0;
      long long issued = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
        const TileCoord tc = decode_tile(p, t, BN);
        if (tc.zero) continue;
        const int za1 = p.a_z1 ? tc.z1 : 0, za2 = p.a_z2 ? tc.z2 : 0;
        const int zb1 = p.b_z1 ? tc.z1 : 0, zb2 = p.b_z2 ? tc.z2 : 0;
        for (int kb = tc.kb0; kb < tc.kb1; ++kb) {
          if (!mbar_wait_bounded(&empty_bar[stage], phase ^ 1, &abort_flag, p.err, kErrTimeoutProducer)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full_bar[stage], Cfg::STAGE_BYTES);
          uint8_t* a_dst = sA + stage * Cfg::A_BYTES;
          uint8_t* b_dst = sB + stage * Cfg::B_BYTES;
          const int k0 = kb * 64;
          if constexpr (A_MN) {
            tma_load_4d(a_dst, &p.ta, &full_bar[stage], tc.m0, k0, za1, za2);
            tma_load_4d(a_dst + 8192, &p.ta, &full_bar[stage], tc.m0 + 64, k0, za1, za2);
          } else {
            tma_load_4d(a_dst, &p.ta, &full_bar[stage], k0, tc.m0, za1, za2);
          }
          if constexpr (B_MN) {
#pragma unroll
            for (int i = 0; i < BN / 64; ++i)
              tma_load_4d(b_dst + i * 8192, &p.tb, &full_bar[stage], tc.n0 + 64 * i, k0, zb1, zb2);
          } else {
            tma_load_4d(b_dst, &p.tb, &full_bar[stage], k0, tc.n0, zb1, zb2);
          }
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok) {
        // Drain: wait (bounded, ignoring the abort flag) for the loads still in flight.
        int dummy_abort = 0;
        const long long inflight = issued < STAGES ? issued : STAGES;
        int s = stage;
        uint32_t ph = phase;
        for (long long i = 0; i < inflight; ++i) {
          if (--s < 0) {
            s = STAGES - 1;
            ph ^= 1;
          }
          mbar_wait_bounded(&full_bar[s], ph, (volatile int*)&dummy_abort, p.err, kErrTimeoutDrain);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------ MMA issuer
      constexpr uint32_t idesc = make_idesc_bf16(128, BN, A_MN, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
        const TileCoord tc = decode_tile(p, t, BN);
        if (tc.zero) continue;
        if (!mbar_wait_bounded(&tempty_bar[acc], acc_phase ^ 1, &abort_flag, p.err, kErrTimeoutMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = tc.kb0; kb < tc.kb1; ++kb) {
          if (!mbar_wait_bounded(&full_bar[stage], phase, &abort_flag, p.err, kErrTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(sA + stage * Cfg::A_BYTES);
          const uint32_t b_base = smem_u32(sB + stage * Cfg::B_BYTES);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint64_t ad = A_MN ? make_sdesc_sw128(a_base + kk * 2048, 8192, 1024)
                                     : make_sdesc_sw128(a_base + kk * 32, 16, 1024);
            const uint64_t bd = B_MN ? make_sdesc_sw128(b_base + kk * 2048, 8192, 1024)
                                     : make_sdesc_sw128(b_base + kk * 32, 16, 1024);
            umma_bf16(d_tmem, ad, bd, idesc, (kb > tc.kb0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(&empty_bar[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit(&tfull_bar[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
      // Wait for every MMA this thread issued before TMEM can be released.
      umma_commit(&drain_bar);
      int dummy_abort = 0;
      mbar_wait_bounded(&drain_bar, 0, (volatile int*)&dummy_abort, p.err, kErrTimeoutDrain);
    }
  } else {
    // ------------------------------------------------ epilogue (warps 2..)
    const int ew = warp - 2;    // 0..NEPI-1
    const int quad = warp & 3;  // TMEM lane quadrant this warp may access
    const int half = ew >> 2;   // column group of the tile
    const int r_local = quad * 32 + lane;
    if constexpr (KIND >= 2) {
      tma_epilogue_loop<BN, EPI, KIND, false>(p, total, blockIdx.x, gridDim.x, 0, sEpi, aux_bar, tfull_bar,
                                              tempty_bar, 0u, 0u, true, tmem_base, &abort_flag, warp, lane);
    } else {
    uint8_t* buf0 = sEpi + ew * 2 * kStageTileBytes;
    uint8_t* buf1 = buf0 + kStageTileBytes;
    // Columns this warp owns: half of the tile (for BN = 64 with staging, warps of the
    // second half idle: a staged chunk is 64 columns wide).
    constexpr int COLS = STAGED ? (BN >= 128 ? BN / 2 : (BN == 64 ? 64 : 0)) : BN / 2;
    const bool active = !(STAGED && BN == 64 && half == 1);
    const int col_off = STAGED && BN == 64 ? 0 : half * (BN / 2);
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x; t < total; t += gridDim.x) {
      const TileCoord tc = decode_tile(p, t, BN);
      const int row = tc.m0 + r_local;
      if (tc.zero) {
        if constexpr (STAGED) {
          if (active)
            for (int c = 0; c < COLS; c += 64) epilogue_zero64<EPI>(p, tc, tc.m0 + quad * 32, tc.n0 + col_off + c, lane);
        } else {
          for (int c = 0; c < COLS; c += 32) epilogue_zero_chunk<EPI>(p, tc, row, tc.n0 + col_off + c);
        }
        continue;
      }
      if (!mbar_wait_bounded(&tfull_bar[acc], acc_phase, &abort_flag, p.err, kErrTimeoutEpilogue)) break;
      tc_fence_after();
      const uint32_t t_addr = tmem_base + ((uint32_t)(quad * 32) << 16) + acc * BN + col_off;
      if constexpr (STAGED) {
        if (active) {
#pragma unroll 1
          for (int c = 0; c < COLS; c += 64) {
            float v[64];
            tmem_ld64(t_addr + c, v);
            epilogue_chunk64<EPI>(p, tc, v, tc.m0 + quad * 32, tc.n0 + col_off + c, buf0, buf1, lane);
          }
        }
      } else {
#pragma unroll 1
        for (int c = 0; c < COLS; c += 32) {
          float v[32];
          tmem_ld32(t_addr + c, v);
          epilogue_chunk<EPI>(p, tc, v, row, tc.n0 + col_off + c);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty_bar[acc]);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
  }

    }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
}

}  // namespace bd
