// dK + dV from materialised P and dS (CTA pairs, cta_group::2).
//
// Replaces the reference's packed dK/dV launch (flash_attn/attention.py:
// 1602-1620) when the dQ kernel has written P and dS to a workspace (see
// KParams::ws). The reference's kernel recomputes S = Q K^T and dP = dO V^T
// for every (key tile, query block); here they were computed once, by the dQ
// kernel, so this kernel is two accumulations per (query tile, key tile):
//
//   dV[k rows] += P^T dO      dK[k rows] += dS^T Q      (dK scaled at the end)
//
// A pair owns 128 key rows (64 per CTA). Both fp32 accumulators stay in TMEM
// for the whole kernel: dK in columns [0, D/2), dV in [D/2, D) of each CTA, in
// the 2x2 layout of attn_pair_kernel.cuh. P^T and dS^T are read as MN-major A
// operands straight from the workspace's [128 queries][256 keys] blocks (a TMA
// box of 64 keys x 128 queries per CTA); Q and dO are MN-major B operands
// split along head_dim between the two CTAs, as in the other pair kernels.
//
// Ring stages are 32 KB = two 16 KB panels under one barrier (half the
// barrier waits and commits of 16 KB stages for the single issuing thread).
// Per query tile ("sub-item") the ring carries 1 + 2 * D/256 stages in this
// order: [dS^T | P^T], then for g = 0 .. D/256-1 the two 64-column panels of
// Q and then of dO for head_dim columns 256g + 128 * rank + [0, 128). The A
// stage is held for the whole sub-item, the B stages are released as they
// are consumed. Every wait is bounded as elsewhere.
#pragma once
#include "attn_kernel.cuh"

namespace gqafa {

template <int D_, int NSTAGES_, bool BF16_>
struct DkvCfg {
  static constexpr int D = D_, NSTAGES = NSTAGES_;
  static constexpr bool BF16 = BF16_;
  static constexpr bool PAIR = true;
  static constexpr bool ROWS_ARE_Q = false;
  static constexpr int NCHUNK = 1;
  static constexpr int M = 64, MP = 128;
  static constexpr int BN = 256;            // query rows per item (two 128-row query tiles)
  static constexpr int NACC = D / 256;      // N=256 pair instructions per accumulator and k-step
  static constexpr int ACC_COLS = D / 2;    // TMEM columns of one accumulator per CTA
  static constexpr int PANEL_BYTES = 128 * 128;      // 128 rows x 64 columns, 16-bit
  static constexpr int STAGE_BYTES = 2 * PANEL_BYTES;
  static constexpr int SUB_STAGES = 1 + 2 * NACC;
  static constexpr int Y_BOX = 128;
  static constexpr int NBARS = 2 * NSTAGES + 1;
  static constexpr int SMEM_BYTES = 1024 + NSTAGES * STAGE_BYTES + NBARS * 8 + 16;
  static constexpr uint32_t IDESC = make_idesc(MP, 256, BF16, true, true);

  static_assert(D % 256 == 0 && 2 * ACC_COLS <= 512, "dK and dV accumulators in TMEM");
  static_assert(NSTAGES >= SUB_STAGES, "ring");
  static_assert(SMEM_BYTES <= 232448, "shared memory");
};

template <class C>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(256, 1)
    attn_dkv_kernel(const __grid_constant__ CUtensorMap tmWS, const __grid_constant__ CUtensorMap tmQ,
                    const __grid_constant__ CUtensorMap tmDO, const KParams p) {
  constexpr int M = C::M, MP = C::MP, NST = C::NSTAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sRing = smem;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sRing + NST * C::STAGE_BYTES);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + C::NBARS);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const uint32_t bar0 = smem_u32(bars);
  auto BAR_FULL = [&](int s) { return bar0 + 8u * s; };
  auto BAR_EMPTY = [&](int s) { return bar0 + 8u * (NST + s); };
  const uint32_t BAR_FINAL = bar0 + 8u * (2 * NST);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = (rank == 0);

  // ---- tile decode: one pair per (key tile, KV head, batch), heaviest first
  int idx = blockIdx.x >> 1;
  const int h = idx % p.Hkv;
  idx /= p.Hkv;
  const int b = idx % p.B;
  idx /= p.B;
  const int tile = p.tile_begin + idx;
  const int pr0 = tile * MP;
  const int r0 = pr0 + M * static_cast<int>(rank);
  const int N = p.N, G = p.G;
  const int T = (N + 127) / 128;
  const bool swa = p.causal && p.window > 0;
  // Query tiles whose rows can attend this pair's keys.
  const int t_lo = p.causal ? pr0 / 128 : 0;
  const int t_hi = swa ? min(T, (pr0 + MP - 1 + p.window - 1) / 128 + 1) : T;
  const int kblk = pr0 / 256;                        // key block of the workspace
  const int kcol = (pr0 % 256) + M * static_cast<int>(rank);  // this CTA's 64 keys within it
  // Does query tile t have a stored block for key block kblk?
  auto stored = [&](int t) {
    int jlo, jn;
    ws_key_blocks(t, N, p.causal, p.window, jlo, jn);
    return kblk >= jlo && kblk < jlo + jn;
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < NST; ++s) {
      mbar_init(BAR_FULL(s), 1);
      mbar_init(BAR_EMPTY(s), 1);
    }
    mbar_init(BAR_FINAL, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmWS);
    prefetch_tmap(&tmQ);
    prefetch_tmap(&tmDO);
  }
  if (warp == 1) {
    tmem_alloc_pair(smem_u32(tmem_slot), 512);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;

  if (warp == 0) {
    // ======================= TMA producer (both CTAs) =======================
    if (lane == 0 && !p.no_loads) {
      bool ok = true;
      uint32_t cnt = 0;
      auto acquire = [&](int& st) -> bool {
        st = cnt % NST;
        const uint32_t ph = (cnt / NST) & 1u;
        if (!mbar_wait_cluster(BAR_EMPTY(st), ph ^ 1u, abort_flag, p.status, ST_TIMEOUT_RING_EMPTY, p.wait_limit)) return false;
        if (leader) mbar_arrive_expect_tx(BAR_FULL(st), 2 * C::STAGE_BYTES);
        ++cnt;
        return true;
      };
      // P / dS blocks are read once (evict-first); Q and dO tiles are read by
      // every key tile of the group (evict-last).
      const uint64_t pol_ws = l2_policy_evict_first(), pol_qdo = l2_policy_evict_last();
      // Sub-items in the order (query tile t descending, query head g0): all
      // pairs of a KV group start at the last query tile and walk down
      // together, so concurrent pairs read the same Q / dO tiles from L2.
      long long before = ws_blocks_before(t_hi, N, p.causal, p.window);  // blocks of tiles < t_hi
      for (int t = t_hi - 1; t >= t_lo && ok; --t) {
        int jlo, jn;
        ws_key_blocks(t, N, p.causal, p.window, jlo, jn);
        before -= jn;  // now: blocks of tiles < t
        if (!(kblk >= jlo && kblk < jlo + jn)) continue;
        for (int g0 = 0; g0 < G && ok; ++g0) {
          const int hq = h * G + g0;
          const long long blk = (static_cast<long long>(b) * p.Hq + hq) * p.ws_bph + before + (kblk - jlo);
          int st;
          // [dS^T | P^T]: 128 queries x this CTA's 64 keys of the block, each
          ok = acquire(st);
          if (!ok) break;
          const uint32_t full_l = mapa_shared(BAR_FULL(st), 0);
          tma_load_3d_pair_hint(smem_u32(sRing + st * C::STAGE_BYTES), &tmWS, full_l, kcol, 0,
                                static_cast<int>(p.ws_blocks + blk), pol_ws);
          tma_load_3d_pair_hint(smem_u32(sRing + st * C::STAGE_BYTES + C::PANEL_BYTES), &tmWS, full_l, kcol, 0,
                                static_cast<int>(blk), pol_ws);
          for (int g = 0; g < C::NACC && ok; ++g) {
            for (int m = 0; m < 2 && ok; ++m) {
              const CUtensorMap* map = (m == 0) ? &tmQ : &tmDO;
              ok = acquire(st);
              if (!ok) break;
              const uint32_t fl = mapa_shared(BAR_FULL(st), 0);
              for (int j = 0; j < 2; ++j)
                tma_load_4d_pair_hint(smem_u32(sRing + st * C::STAGE_BYTES + j * C::PANEL_BYTES), map, fl,
                                      64 * (4 * g + 2 * static_cast<int>(rank) + j), 128 * t, hq, b, pol_qdo);
            }
          }
        }
      }
    }
  } else if (warp == 1) {
    // ======================= MMA issuer (leader CTA only) =======================
    if (leader && lane == 0) {
      bool ok = true;
      uint32_t cnt = 0;
      bool first = true;
      const uint64_t dRing = sw128_desc(smem_u32(sRing), C::PANEL_BYTES, 1024);
      auto full = [&](uint32_t c) {
        return mbar_wait_cluster(BAR_FULL(c % NST), (c / NST) & 1u, abort_flag, p.status, ST_TIMEOUT_RING_FULL, p.wait_limit);
      };
      auto sdesc = [&](uint32_t c) { return dRing + static_cast<uint64_t>(((c % NST) * C::STAGE_BYTES) >> 4); };
      for (int t = t_hi - 1; t >= t_lo && ok; --t) {
        if (!stored(t)) continue;
        for (int g0 = 0; g0 < G && ok; ++g0) {
          const uint32_t cA = cnt;  // [dS^T | P^T]
          ok = full(cA);
          if (!ok) break;
          tc_fence_after();
          const uint64_t aDS = sdesc(cA), aP = aDS + static_cast<uint64_t>(C::PANEL_BYTES >> 4);
#pragma unroll 1
          for (int g = 0; g < C::NACC && ok; ++g) {
#pragma unroll 1
            for (int m = 0; m < 2; ++m) {
              const uint32_t c2 = cA + 1 + 2 * g + m;
              ok = full(c2);
              if (!ok) break;
              tc_fence_after();
              const uint64_t a = (m == 0) ? aDS : aP;
              const uint64_t yb = sdesc(c2);
              const uint32_t acc = m * C::ACC_COLS + 128u * g;
#pragma unroll
              for (int tt = 0; tt < 8; ++tt) {
                const uint64_t off = static_cast<uint64_t>((tt * 2048) >> 4);
                mma_ss_pair(tbase + acc, a + off, yb + off, C::IDESC, (first && tt == 0) ? 0u : 1u);
              }
              mma_commit_pair(BAR_EMPTY(c2 % NST));
            }
          }
          if (!ok) break;
          first = false;
          mma_commit_pair(BAR_EMPTY(cA % NST));
          cnt += C::SUB_STAGES;
        }
      }
      if (ok) mma_commit_pair(BAR_FINAL);
    }
  } else if (warp >= 4) {
    // ======================= epilogue warps (both CTAs) =======================
    const int q4 = warp & 3;
    const int half = q4 >> 1;
    const int row = 32 * (q4 & 1) + lane;
    const uint32_t tq = tbase + (static_cast<uint32_t>(q4 * 32) << 16);
    bool any = false;
    for (int t = t_lo; t < t_hi && !any; ++t) any = stored(t);
    bool ok = true;
    if (any) {
      ok = mbar_wait_cluster(BAR_FINAL, 0, abort_flag, p.status, ST_TIMEOUT_ACC, p.wait_limit);
      ok = __all_sync(0xffffffffu, ok);
      if (ok) tc_fence_after();
    }
    const int orow = r0 + row;
    // tcgen05.ld is warp-collective: every lane loads, only live rows store.
    if (ok) {
#pragma unroll 1
      for (int m = 0; m < 2; ++m) {
        void* out = (m == 0) ? p.out : p.out2;
        const long long obase = (m == 0)
                                    ? static_cast<long long>(b) * p.out_sb + static_cast<long long>(h) * p.out_sh +
                                          static_cast<long long>(orow) * p.out_sn
                                    : static_cast<long long>(b) * p.out2_sb + static_cast<long long>(h) * p.out2_sh +
                                          static_cast<long long>(orow) * p.out2_sn;
        const float mul = (m == 0) ? p.scale : 1.f;
#pragma unroll 1
        for (int g = 0; g < C::NACC; ++g) {
#pragma unroll 1
          for (int k = 0; k < 4; ++k) {
            float v[32];
            if (any) {
              uint32_t r[32];
              tmem_ld32(tq + C::ACC_COLS * m + g * 128 + 32 * k, r);
#pragma unroll
              for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]) * mul;
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j) v[j] = 0.f;
            }
            if (orow < N) store_out32<C::BF16>(out, obase + 256 * g + 128 * half + 32 * k, v, p.out_f32 != 0);
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync_all();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tbase, 512);
  }
}

}  // namespace gqafa
