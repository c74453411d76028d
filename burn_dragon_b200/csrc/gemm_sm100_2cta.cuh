// gemm_sm100_2cta.cuh — the tcgen05 engine on CTA pairs (cta_group::2), 256-row tiles.
//
// A cluster of two CTAs on neighbouring SMs computes one 256 x BN tile: each CTA stages
// its own 128 rows of A and its own half (BN/2 rows) of B, the even ("leader") CTA
// issues tcgen05.mma.cta_group::2 (M = 256) which reads the operands of both CTAs and
// writes a 128 x BN fp32 accumulator into each CTA's TMEM. Per SM this halves the B
// bytes per FLOP of the 1-CTA 128 x BN tile — the operand traffic that limits the
// MMA-bound BDH contractions (weight gradients, causal scores, decoder products).
//
//   both CTAs  warp 0     TMA producer: own A rows + own B half; completion counted on
//                         the leader's full barrier (cta_group::2 loads, no multicast)
//   leader     warp 1     TMEM (pair allocation) + single-thread MMA issuer; commits
//                         multicast to both CTAs' empty / tmem-full barriers
//   both CTAs  warps 2-9  epilogue on their own 128 rows; release the accumulator on
//                         the leader's tmem-empty barrier (one arrival per epilogue warp of both CTAs)
// All epilogue kinds: fp32, staged bf16 and the TMA epilogues (each CTA runs the same
// per-warp TMA epilogue loop as the 1-CTA kernel on its own 128 rows). For the
// TMA-epilogue modes the pair runs 256 x 256 tiles (each CTA 128 x 256, two 64-column
// chunks per epilogue warp): per output element a CTA then stages half the operand bytes
// of a 1-CTA 128 x 128 tile. (256 x 128 pair tiles measured 25-45% slower than the 1-CTA
// kernel: the saving is smaller and the pair couples two CTAs' epilogues.)
// Bounded waits as in the 1-CTA kernel.
#pragma once

namespace bd {

template <int BN, int KIND>
struct Gemm2Cfg {
  static constexpr int A_BYTES = 128 * 64 * 2;
  static constexpr int B_BYTES = (BN / 2) * 64 * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  // TMA-epilogue kinds: the 1-CTA kernel's warp counts and tile buffers (GemmCfg)
  static constexpr int NEPI = GemmCfg<BN, KIND>::NEPI;
  static constexpr int EPI_BYTES = KIND >= 2 ? GemmCfg<BN, KIND>::EPI_BYTES : (KIND == 1 ? 8 * 2 * 4096 : 0);
  // TMA-epilogue kinds with BN = 256 stage 32 KB per CTA per k-block: one stage fewer
  // keeps the ring plus the epilogue tile buffers inside 227 KB
  static constexpr int STAGES = KIND == 4   ? (BN == 256 ? 4 : 5)
                                : KIND >= 2 ? (BN == 256 ? 3 : 4)
                                : KIND == 1 ? (BN == 256 ? 5 : 6)
                                            : (BN == 256 ? 6 : 8);
  static constexpr int SMEM = STAGES * STAGE_BYTES + EPI_BYTES + 1024;
  static constexpr int TMEM_COLS = 2 * BN;
  static constexpr int THREADS = 64 + 32 * NEPI;
};

template <int BN, bool A_MN, bool B_MN, int EPI>
__global__ void __launch_bounds__(Gemm2Cfg<BN, epi_kind<EPI>()>::THREADS, 1)
    gemm_sm100_2cta_kernel(const __grid_constant__ GemmParams p) {
  constexpr int KIND = epi_kind<EPI>();
  static_assert(KIND < 2 || BN == 128 || BN == 256, "the TMA epilogue is built for tile N = 128 / 256");
  constexpr bool STAGED = KIND == 1;
  using Cfg = Gemm2Cfg<BN, KIND>;
  constexpr int STAGES = Cfg::STAGES;
  constexpr int HB = BN / 2;  // B rows staged by each CTA
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
  const uint32_t crank = cluster_ctarank();
  const bool leader = crank == 0;
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
      mbar_init(&tempty_bar[a], 2 * Cfg::NEPI);
    }
    mbar_init(&drain_bar, 1);
    for (int w = 0; w < Cfg::NEPI; ++w)
      for (int b = 0; b < 3; ++b) mbar_init(&aux_bar[w][b], 1);
    fence_barrier_init();
    tma_prefetch_desc(&p.ta);
    tma_prefetch_desc(&p.tb);
  }
  if (warp == 1) tmem_alloc_pair(&tmem_base_s, Cfg::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // the peer's barriers exist before any remote arrive / complete_tx
  tc_fence_after();
  const uint32_t tmem_base = tmem_base_s;

  const int total = p.tiles_m * p.tiles_n * p.splits * p.Z1 * p.Z2;
  const int cluster_id = blockIdx.x >> 1;
  const int n_clusters = gridDim.x >> 1;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------ TMA producer (both CTAs)
      int stage = 0;
      uint32_t phase = 0;
      long long issued = 0;
      bool ok = true;
      for (int t = cluster_id; t < total && ok; t += n_clusters) {
        const TileCoord tc = decode_tile_pair(p, t, BN);
        if (tc.zero) continue;
        const int za1 = p.a_z1 ? tc.z1 : 0, za2 = p.a_z2 ? tc.z2 : 0;
        const int zb1 = p.b_z1 ? tc.z1 : 0, zb2 = p.b_z2 ? tc.z2 : 0;
        const int am0 = tc.m0 + 128 * (int)crank;
        const int bn0 = tc.n0 + HB * (int)crank;
        for (int kb = tc.kb0; kb < tc.kb1; ++kb) {
          if (!mbar_wait_bounded(&empty_bar[stage], phase ^ 1, &abort_flag, p.err, kErrTimeoutProducer)) {
            ok = false;
            break;
          }
          if (leader) mbar_arrive_expect_tx(&full_bar[stage], 2 * Cfg::STAGE_BYTES);
          uint8_t* a_dst = sA + stage * Cfg::A_BYTES;
          uint8_t* b_dst = sB + stage * Cfg::B_BYTES;
          const int k0 = kb * 64;
          if constexpr (A_MN) {
            tma_load_4d_pair(a_dst, &p.ta, &full_bar[stage], am0, k0, za1, za2);
            tma_load_4d_pair(a_dst + 8192, &p.ta, &full_bar[stage], am0 + 64, k0, za1, za2);
          } else {
            tma_load_4d_pair(a_dst, &p.ta, &full_bar[stage], k0, am0, za1, za2);
          }
          if constexpr (B_MN) {
#pragma unroll
            for (int i = 0; i < HB / 64; ++i)
              tma_load_4d_pair(b_dst + i * 8192, &p.tb, &full_bar[stage], bn0 + 64 * i, k0, zb1, zb2);
          } else {
            tma_load_4d_pair(b_dst, &p.tb, &full_bar[stage], k0, bn0, zb1, zb2);
          }
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok && leader) {
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
    if (lane == 0 && leader) {
      // ------------------------------------------------ MMA issuer (leader only)
      constexpr uint32_t idesc = make_idesc_bf16(256, BN, A_MN, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int t = cluster_id; t < total && ok; t += n_clusters) {
        const TileCoord tc = decode_tile_pair(p, t, BN);
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
            umma_bf16_pair(d_tmem, ad, bd, idesc, (kb > tc.kb0 || kk > 0) ? 1u : 0u);
          }
          umma_commit_pair(&empty_bar[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit_pair(&tfull_bar[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
      umma_commit_pair(&drain_bar);
      int dummy_abort = 0;
      mbar_wait_bounded(&drain_bar, 0, (volatile int*)&dummy_abort, p.err, kErrTimeoutDrain);
    }
  } else if constexpr (KIND >= 2) {
    // ------------------------------------------------ TMA epilogue (both CTAs, own 128 rows)
    tma_epilogue_loop<BN, EPI, KIND, true>(p, total, cluster_id, n_clusters, 128 * (int)crank, sEpi, aux_bar,
                                           tfull_bar, tempty_bar, map_to_cta(&tempty_bar[0], 0),
                                           map_to_cta(&tempty_bar[1], 0), leader, tmem_base, &abort_flag, warp, lane);
  } else {
    // ------------------------------------------------ epilogue (both CTAs, own 128 rows)
    const int ew = warp - 2;
    const int quad = warp & 3;
    const int half = ew >> 2;
    const int r_local = quad * 32 + lane;
    uint8_t* buf0 = sEpi + ew * 2 * kStageTileBytes;
    uint8_t* buf1 = buf0 + kStageTileBytes;
    constexpr int COLS = STAGED ? (BN >= 128 ? BN / 2 : 64) : BN / 2;
    const bool active = !(STAGED && BN == 64 && half == 1);
    const int col_off = STAGED && BN == 64 ? 0 : half * (BN / 2);
    const uint32_t leader_tempty0 = map_to_cta(&tempty_bar[0], 0);
    const uint32_t leader_tempty1 = map_to_cta(&tempty_bar[1], 0);
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = cluster_id; t < total; t += n_clusters) {
      TileCoord tc = decode_tile_pair(p, t, BN);
      tc.m0 += 128 * (int)crank;
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
      if (lane == 0) {
        if (leader)
          mbar_arrive(&tempty_bar[acc]);
        else
          mbar_arrive_cluster(acc ? leader_tempty1 : leader_tempty0);
      }
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // the leader's MMAs (into both CTAs' TMEM / smem) are done
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, Cfg::TMEM_COLS);
  }
}

}  // namespace bd
