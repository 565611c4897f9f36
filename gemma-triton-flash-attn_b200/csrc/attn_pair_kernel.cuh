// Head_dim-512 kernels on CTA pairs (cta_group::2).
//
// Same roles and math as attn_kernel.cuh (ROLE_FWD / ROLE_DQ / ROLE_DK /
// ROLE_DV; the reference launches they replace are listed there), but a row
// tile of 128 rows is shared by the two CTAs of a cluster, 64 rows each:
//
//   * every tcgen05.mma is issued by the even CTA (the leader) with
//     cta_group::2 and M = 128: A comes from each CTA's own 64 rows, B is split
//     along N between the two CTAs, and each CTA's TMEM receives its 64 rows;
//   * so each CTA loads only half of every streamed B operand: the score MMAs
//     read BN/2 key (or query) rows per CTA, the accumulate MMAs 128 of every
//     256 head_dim columns per CTA;
//   * the fp32 accumulator of 64 rows x 512 columns takes 256 TMEM columns per
//     CTA (the 2x2 layout: lanes 0-63 hold the first half of each N range,
//     lanes 64-127 the second half), which leaves room for double-buffered
//     score buffers. For the forward this is what removes the 1-CTA kernel's
//     second pass: the whole 512-column O fits, so S is computed once.
//
// Synchronisation across the pair: TMA loads of both CTAs complete on the
// leader's "full" barriers (the leader expects both CTAs' bytes); the
// leader's tcgen05.commit arrives on the "empty", "scores ready" and
// "accumulator done" barriers of both CTAs (multicast commit); the row warps
// of both CTAs arrive on the leader's "P ready" barrier. No TMA multicast is
// used. Every wait is bounded as in attn_kernel.cuh.
#pragma once
#include "attn_kernel.cuh"

namespace gqafa {

// RW_ = number of row warpgroups (4 warps each). With RW_ = 2 two warps share
// every TMEM lane quadrant and split each item's columns between them, so the
// elementwise work per item (exp2, masking, dS, packing into the P buffer) is
// spread over twice as many warps.
template <int ROLE_, int D_, int BN_, int NS_, int NSTAGES_, bool BF16_, int RW_ = 1>
struct PairCfg {
  static constexpr int ROLE = ROLE_, D = D_, BN = BN_, NS = NS_, NSTAGES = NSTAGES_;
  static constexpr int RW = RW_;
  static constexpr int THREADS = 128 + 128 * RW;
  static constexpr bool BF16 = BF16_;
  static constexpr bool PAIR = true;
  static constexpr int M = 64;     // rows per CTA
  static constexpr int MP = 128;   // rows per pair
  static constexpr int NCHUNK = 1;
  static constexpr bool HAS_DP = (ROLE == ROLE_DQ || ROLE == ROLE_DK);
  static constexpr bool ROWS_ARE_Q = (ROLE == ROLE_DQ || ROLE == ROLE_FWD);
  static constexpr int PANELS_D = D / 64;
  static constexpr int R_PANEL = M * 128;
  static constexpr int R_BYTES = PANELS_D * R_PANEL * (HAS_DP ? 2 : 1);
  // Ring stages are 32 KB, one barrier each: two 16 KB panels of 128 rows x
  // 64 columns (fewer barrier waits and commits for the single issuing
  // thread than one panel per stage).
  static constexpr int PANEL_BYTES = 128 * 128;
  static constexpr int STAGE_BYTES = 2 * PANEL_BYTES;
  static constexpr int CR = BN / 2;                     // score-operand rows this CTA loads per item
  static constexpr int C_PANEL_BYTES = CR * 128;
  static constexpr int CP = STAGE_BYTES / C_PANEL_BYTES;  // score-operand panels per stage (2 or 4)
  static constexpr int C_STAGES = PANELS_D / CP;
  static constexpr int C_BOX = CR, Y_BOX = 128;
  static constexpr int NACC = D / 256;                  // N=256 accumulate instructions per k-step
  static constexpr int YH = BN / 128;                   // 128-row halves of an accumulate operand
  // one stage per (instruction g, half hh): this CTA's two 64-column panels of
  // its 128 of every 256 columns
  static constexpr int Y_STAGES = NACC * YH;
  static constexpr int RING_BYTES = NSTAGES * STAGE_BYTES;
  static constexpr int PBUF_ONE = M * BN * 2;
  static constexpr int PBUF_BYTES = NS * PBUF_ONE;
  // dQ / dK with one S / dP buffer: the next item's S MMAs are issued as soon
  // as the row warps have read S ("S free"), ahead of this item's accumulate
  // MMAs, so the tensor pipe works while the row warps form dS.
  static constexpr bool EARLY_S = HAS_DP && NS == 1;
  static constexpr int NBARS = 2 * NSTAGES + 1 + 4 * NS + 2;
  // sRow (M floats), then for the forward the row-statistics exchange between
  // the 2 * RW warps that hold parts of the same rows:
  // [2 slots][2 * RW parts][M] maxima and [2 * RW parts][M] partial sums.
  static constexpr int XCH_FLOATS = (ROLE == ROLE_FWD) ? 6 * RW * M : 0;
  static constexpr int MISC_BYTES = M * 4 + XCH_FLOATS * 4 + NBARS * 8 + 16;
  static constexpr int SMEM_BYTES = 1024 + R_BYTES + RING_BYTES + PBUF_BYTES + MISC_BYTES;
  static constexpr int ACC_COLS = D / 2;
  static constexpr int SBUF_COLS = BN / 2;
  static constexpr uint32_t IDESC_S = make_idesc(MP, BN, BF16, false);
  static constexpr uint32_t IDESC_Y = make_idesc(MP, 256, BF16, true);
  static constexpr int KCH = SBUF_COLS / 32;  // 32-column chunks of an item per TMEM lane
  static constexpr int KCHW = KCH / RW;       // ... per row warp

  static_assert(RW == 1 || RW == 2 || RW == 4, "row warpgroups");
  static_assert(KCH % RW == 0 && (NACC * 4) % RW == 0, "column split");
  static_assert(ROLE != ROLE_FWD || ((ACC_COLS / 32) % (2 * RW) == 0 && KCHW % 2 == 0), "forward column split");

  static_assert(D % 256 == 0, "D");
  static_assert(BN == 128 || BN == 256, "BN");
  static_assert(ACC_COLS + NS * SBUF_COLS * (HAS_DP ? 2 : 1) <= 512, "TMEM");
  static_assert(PANELS_D % CP == 0, "score-operand stages");
  static_assert(SMEM_BYTES <= 232448, "shared memory");
};

template <class C>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(C::THREADS, 1)
    attn_pair_kernel(const __grid_constant__ CUtensorMap tmR1, const __grid_constant__ CUtensorMap tmR2,
                     const __grid_constant__ CUtensorMap tmC1, const __grid_constant__ CUtensorMap tmC2,
                     const __grid_constant__ CUtensorMap tmY, const __grid_constant__ CUtensorMap tmWS,
                     const KParams p) {
  constexpr int M = C::M, MP = C::MP, BN = C::BN, NS = C::NS, NST = C::NSTAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sR1 = smem;
  uint8_t* sR2 = smem + C::PANELS_D * C::R_PANEL;
  uint8_t* sRing = smem + C::R_BYTES;
  uint8_t* sP = sRing + C::RING_BYTES;
  float* sRow = reinterpret_cast<float*>(sP + C::PBUF_BYTES);
  float* sX = sRow + M;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sX + C::XCH_FLOATS);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + C::NBARS);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const uint32_t bar0 = smem_u32(bars);
  auto BAR_FULL = [&](int s) { return bar0 + 8u * s; };
  auto BAR_EMPTY = [&](int s) { return bar0 + 8u * (NST + s); };
  const uint32_t BAR_RFULL = bar0 + 8u * (2 * NST);
  auto BAR_SFULL = [&](int s) { return bar0 + 8u * (2 * NST + 1 + s); };
  auto BAR_PREADY = [&](int s) { return bar0 + 8u * (2 * NST + 1 + NS + s); };
  const uint32_t BAR_ACC = bar0 + 8u * (2 * NST + 1 + 2 * NS);
  // Completes once, after the last accumulate MMA. The epilogue waits on it
  // rather than on BAR_ACC: with two score buffers BAR_ACC can still be two
  // phases short of the end, where its parity is indistinguishable.
  const uint32_t BAR_FINAL = bar0 + 8u * (2 * NST + 2 + 2 * NS);
  // S of the item is in TMEM (dP may still be in flight): lets the row warps
  // compute P while the dP MMAs run (dQ / dK).
  auto BAR_SREADY = [&](int s) { return bar0 + 8u * (2 * NST + 3 + 2 * NS + s); };
  // The row warps of both CTAs have read S of the buffer (EARLY_S).
  auto BAR_SFREE = [&](int s) { return bar0 + 8u * (2 * NST + 3 + 3 * NS + s); };

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool prof = (p.prof != nullptr);
  unsigned long long wc[WC_NUM] = {};
  const long long t_start = prof ? clock64() : 0;
  auto tick = [&]() -> long long { return prof ? clock64() : 0; };
  auto tock = [&](int k, long long t0) {
    if (prof) wc[k] += static_cast<unsigned long long>(clock64() - t0);
  };
  const bool leader = (rank == 0);

  // ---- tile decode (per pair; both CTAs see the same items)
  const int heads = C::ROWS_ARE_Q ? p.Hq : p.Hkv;
  int idx = blockIdx.x >> 1;
  const int h = idx % heads;
  idx /= heads;
  const int b = idx % p.B;
  idx /= p.B;
  const int tile = p.tile_begin + (C::ROWS_ARE_Q ? (p.num_row_tiles - 1 - idx) : idx);
  const int pr0 = tile * MP;
  const int r0 = pr0 + M * static_cast<int>(rank);
  const int N = p.N, G = p.G;
  const bool swa = p.causal && p.window > 0;

  int jlo, jn, n_items;
  if constexpr (C::ROWS_ARE_Q) {
    const int kv_hi = p.causal ? min(p.Nk, pr0 + MP + p.qoff) : p.Nk;
    const int kv_lo = swa ? max(0, pr0 + p.qoff - p.window + 1) : 0;
    jlo = kv_lo / BN;
    jn = (kv_hi + BN - 1) / BN - jlo;
    n_items = jn;
  } else {
    const int q_lo = p.causal ? pr0 : 0;
    const int q_hi = swa ? min(N, pr0 + MP - 1 + p.window) : N;
    jlo = q_lo / BN;
    jn = (q_hi + BN - 1) / BN - jlo;
    n_items = G * jn;
  }
  auto item_col0 = [&](int i) { return (jlo + (C::ROWS_ARE_Q ? i : i % jn)) * BN; };
  auto item_headC = [&](int i) { return C::ROWS_ARE_Q ? h / G : h * G + i / jn; };

  if (threadIdx.x == 0) {
    for (int s = 0; s < NST; ++s) {
      mbar_init(BAR_FULL(s), 1);
      mbar_init(BAR_EMPTY(s), 1);
    }
    mbar_init(BAR_RFULL, 1);
    for (int s = 0; s < NS; ++s) {
      mbar_init(BAR_SFULL(s), 1);
      mbar_init(BAR_SREADY(s), 1);
      mbar_init(BAR_SFREE(s), 8 * C::RW);
      mbar_init(BAR_PREADY(s), 8 * C::RW);  // 4 * RW row warps in each CTA of the pair
    }
    mbar_init(BAR_ACC, 1);
    mbar_init(BAR_FINAL, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmR1);
    prefetch_tmap(&tmC1);
    prefetch_tmap(&tmY);
    if constexpr (C::HAS_DP) {
      prefetch_tmap(&tmR2);
      prefetch_tmap(&tmC2);
    }
  }
  if (warp == 1) {
    tmem_alloc_pair(smem_u32(tmem_slot), 512);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // the peer's barriers are initialised before any cross-CTA arrive
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;

  if (warp == 0) {
    // ======================= TMA producer (both CTAs) =======================
    if (lane == 0 && !p.no_loads) {
      bool ok = true;
      if (leader) mbar_arrive_expect_tx(BAR_RFULL, 2 * C::R_BYTES);
      const uint32_t rfull_l = mapa_shared(BAR_RFULL, 0);
      for (int pn = 0; pn < C::PANELS_D; ++pn)
        tma_load_4d_pair(smem_u32(sR1 + pn * C::R_PANEL), &tmR1, rfull_l, 64 * pn, r0, h, b);
      if constexpr (C::HAS_DP) {
        for (int pn = 0; pn < C::PANELS_D; ++pn)
          tma_load_4d_pair(smem_u32(sR2 + pn * C::R_PANEL), &tmR2, rfull_l, 64 * pn, r0, h, b);
      }
      uint32_t cnt = 0;
      // Acquire the next ring stage; the leader announces both CTAs' bytes.
      auto acquire = [&](int& st) -> bool {
        st = cnt % NST;
        const uint32_t ph = (cnt / NST) & 1u;
        const long long t0 = tick();
        const bool got = mbar_wait_cluster(BAR_EMPTY(st), ph ^ 1u, abort_flag, p.status, ST_TIMEOUT_RING_EMPTY, p.wait_limit);
        tock(WC_PRODUCER_EMPTY, t0);
        if (!got) return false;
        if (leader) mbar_arrive_expect_tx(BAR_FULL(st), 2 * C::STAGE_BYTES);
        ++cnt;
        return true;
      };
      auto load_c = [&](const CUtensorMap* m, int c0, int hc) -> bool {
        for (int s = 0; s < C::C_STAGES; ++s) {
          int st;
          if (!acquire(st)) return false;
          const uint32_t full_l = mapa_shared(BAR_FULL(st), 0);
          for (int pp = 0; pp < C::CP; ++pp)
            tma_load_4d_pair(smem_u32(sRing + st * C::STAGE_BYTES + pp * C::C_PANEL_BYTES), m, full_l,
                             64 * (C::CP * s + pp), c0 + static_cast<int>(rank) * C::CR, hc, b);
        }
        return true;
      };
      auto load_scores = [&](int i) -> bool {
        const int c0 = item_col0(i), hc = item_headC(i);
        if (!load_c(&tmC1, c0, hc)) return false;
        if constexpr (C::HAS_DP) {
          if (!load_c(&tmC2, c0, hc)) return false;
        }
        return true;
      };
      auto load_y = [&](int i) -> bool {
        const int c0 = item_col0(i), hc = item_headC(i);
        // stage order: [instruction g][128-row half hh]; a stage holds panels
        // j = 0, 1 PANEL_BYTES apart, which is the MN-major operand's LBO.
        for (int g = 0; g < C::NACC; ++g)
          for (int hh = 0; hh < C::YH; ++hh) {
            int st;
            if (!acquire(st)) return false;
            const uint32_t fl = mapa_shared(BAR_FULL(st), 0);
            for (int j = 0; j < 2; ++j)
              tma_load_4d_pair(smem_u32(sRing + st * C::STAGE_BYTES + j * C::PANEL_BYTES), &tmY, fl,
                               64 * (4 * g + 2 * static_cast<int>(rank) + j), c0 + 128 * hh, hc, b);
          }
        return true;
      };
      if constexpr (C::EARLY_S) {
        // the issuer's order: S(0) dP(0), then per item S(i+1), acc(i), dP(i+1)
        auto load_s = [&](int i) { return load_c(&tmC1, item_col0(i), item_headC(i)); };
        auto load_dp = [&](int i) { return load_c(&tmC2, item_col0(i), item_headC(i)); };
        if (n_items > 0) ok = load_s(0) && load_dp(0);
        for (int i = 0; i < n_items && ok; ++i) {
          if (i + 1 < n_items) ok = load_s(i + 1);
          ok = ok && load_y(i);
          if (ok && i + 1 < n_items) ok = load_dp(i + 1);
        }
      } else {
        for (int s = 0; s < NS && s < n_items && ok; ++s) ok = load_scores(s);
        for (int i = 0; i < n_items && ok; ++i) {
          ok = load_y(i);
          if (ok && i + NS < n_items) ok = load_scores(i + NS);
        }
      }
    }
  } else if (warp == 1) {
    // ======================= MMA issuer (leader CTA only) =======================
    if (leader && lane == 0) {
      bool ok = mbar_wait_cluster(BAR_RFULL, 0, abort_flag, p.status, ST_TIMEOUT_RESIDENT, p.wait_limit);
      tc_fence_after();
      const uint32_t aR1 = smem_u32(sR1), aR2 = smem_u32(sR2), aRing = smem_u32(sRing), aP = smem_u32(sP);
      uint32_t cnt = 0;
      // Descriptors are built once; per instruction only the start-address
      // field changes (byte offset >> 4 added to the low bits). Keeping the
      // issuing thread's work per MMA to a few integer adds matters: a 128-row
      // pair MMA with N=128 occupies the tensor pipe for only ~32 cycles.
      const uint64_t dR1 = sw128_desc(aR1, 16, 1024), dR2 = sw128_desc(aR2, 16, 1024);
      const uint64_t dRingK = sw128_desc(aRing, 16, 1024);
      const uint64_t dRingMN = sw128_desc(aRing, C::PANEL_BYTES, 1024);
      const uint64_t dP = sw128_desc(aP, 16, 1024);
      auto scores_from = [&](uint64_t dR, uint32_t d_tmem) -> bool {
#pragma unroll
        for (int s = 0; s < C::C_STAGES; ++s) {
          const int st = cnt % NST;
          const long long t0 = tick();
          const bool got = mbar_wait_cluster(BAR_FULL(st), (cnt / NST) & 1u, abort_flag, p.status, ST_TIMEOUT_RING_FULL, p.wait_limit);
          tock(WC_MMA_FULL_SCORES, t0);
          if (!got) return false;
          tc_fence_after();
          const uint64_t bst = dRingK + static_cast<uint64_t>((st * C::STAGE_BYTES) >> 4);
#pragma unroll
          for (int pp = 0; pp < C::CP; ++pp) {
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const uint64_t ad = dR + static_cast<uint64_t>(((C::CP * s + pp) * C::R_PANEL + 32 * k) >> 4);
              const uint64_t bd = bst + static_cast<uint64_t>((pp * C::C_PANEL_BYTES + 32 * k) >> 4);
              mma_ss_pair(d_tmem, ad, bd, C::IDESC_S, (s | pp | k) != 0);
            }
          }
          mma_commit_pair(BAR_EMPTY(st));
          ++cnt;
        }
        return true;
      };
      auto issue_scores = [&](int i) -> bool {
        const int sb = i % NS;
        if (!scores_from(dR1, tbase + C::ACC_COLS + sb * C::SBUF_COLS)) return false;
        if constexpr (C::HAS_DP) {
          mma_commit_pair(BAR_SREADY(sb));
          if (!scores_from(dR2, tbase + C::ACC_COLS + (NS + sb) * C::SBUF_COLS)) return false;
        }
        mma_commit_pair(BAR_SFULL(sb));
        return true;
      };
      auto issue_acc = [&](int i) -> bool {
        const int sb = i % NS;
        long long t0 = tick();
        if (!mbar_wait_cluster(BAR_PREADY(sb), (i / NS) & 1u, abort_flag, p.status, ST_TIMEOUT_PREADY, p.wait_limit))
          return false;
        tock(WC_MMA_PREADY, t0);
        // Accumulate operand stages (both panels of one instruction g and
        // 128-row half hh) are released right after their MMAs, so an item never
        // needs more ring stages at once than the ring has.
        const uint64_t pb = dP + static_cast<uint64_t>((sb * C::PBUF_ONE) >> 4);
        const uint32_t acc0 = (i > 0) ? 1u : 0u;
#pragma unroll
        for (int g = 0; g < C::NACC; ++g) {
#pragma unroll
          for (int hh = 0; hh < C::YH; ++hh) {
            const uint32_t c2 = cnt + g * C::YH + hh;
            t0 = tick();
            if (!mbar_wait_cluster(BAR_FULL(c2 % NST), (c2 / NST) & 1u, abort_flag, p.status, ST_TIMEOUT_RING_FULL, p.wait_limit))
              return false;
            tock(WC_MMA_FULL_Y, t0);
            tc_fence_after();
            const uint64_t yb = dRingMN + static_cast<uint64_t>(((c2 % NST) * C::STAGE_BYTES) >> 4);
#pragma unroll
            for (int tt = 0; tt < 8 && hh * 8 + tt < BN / 16; ++tt) {
              const int t = hh * 8 + tt;
              const uint64_t ad = pb + static_cast<uint64_t>(((t / 4) * (M * 128) + (t % 4) * 32) >> 4);
              mma_ss_pair(tbase + g * 128, ad, yb + static_cast<uint64_t>((tt * 2048) >> 4), C::IDESC_Y,
                          t > 0 ? 1u : acc0);
            }
            mma_commit_pair(BAR_EMPTY(c2 % NST));
          }
        }
        mma_commit_pair(BAR_ACC);
        cnt += C::Y_STAGES;
        return true;
      };
      if constexpr (C::EARLY_S) {
        auto issue_s = [&](int i) -> bool {
          if (!scores_from(dR1, tbase + C::ACC_COLS)) return false;
          mma_commit_pair(BAR_SREADY(0));
          return true;
        };
        auto issue_dp = [&](int i) -> bool {
          if (!scores_from(dR2, tbase + C::ACC_COLS + C::SBUF_COLS)) return false;
          mma_commit_pair(BAR_SFULL(0));
          return true;
        };
        if (n_items > 0) ok = issue_s(0) && issue_dp(0);
        for (int i = 0; i < n_items && ok; ++i) {
          if (i + 1 < n_items) {
            const long long t0 = tick();
            ok = mbar_wait_cluster(BAR_SFREE(0), i & 1u, abort_flag, p.status, ST_TIMEOUT_PREADY, p.wait_limit);
            tock(WC_MMA_PREADY, t0);
            if (ok) {
              tc_fence_after();
              ok = issue_s(i + 1);
            }
          }
          // dP(i+1) overwrites dP(i), which the row warps have read once they
          // signal P ready for item i (issue_acc waits for that).
          ok = ok && issue_acc(i);
          if (ok && i + 1 < n_items) ok = issue_dp(i + 1);
        }
      } else {
        for (int s = 0; s < NS && s < n_items && ok; ++s) ok = issue_scores(s);
        for (int i = 0; i < n_items && ok; ++i) {
          ok = issue_acc(i);
          if (ok && i + NS < n_items) ok = issue_scores(i + NS);
        }
      }
      if (ok) mma_commit_pair(BAR_FINAL);
    }
  } else if (warp >= 4) {
    // ======================= row warps (both CTAs) =======================
    // 2x2 TMEM layout: lane l of quadrant q holds row 32*(q%2)+l, and the
    // first (q < 2) or second (q >= 2) half of each N range.
    // With RW = 2, warps w and w + 4 share a quadrant; `cs` selects which
    // KCHW of the KCH column chunks (and which part of the epilogue) a warp owns.
    const int rwi = warp - 4;
    const int q4 = warp & 3;
    const int cs = rwi >> 2;
    const int half = q4 >> 1;
    const int row = 32 * (q4 & 1) + lane;
    const uint32_t tq = tbase + (static_cast<uint32_t>(q4 * 32) << 16);
    constexpr int RW = C::RW, KCHW = C::KCHW;
    const int kc0 = cs * KCHW;  // first column chunk this warp owns
    const float LOG2E = 1.4426950408889634f;
    const float sl2 = p.scale_log2;
    bool ok = true;
    float row_lse2 = 0.f, row_delta = 0.f;
    const long long rowbase_q = (static_cast<long long>(b) * p.Hq + (C::ROWS_ARE_Q ? h : 0)) * N;
    const uint32_t pready_l0 = mapa_shared(BAR_PREADY(0), 0);
    const uint32_t sfree_l0 = mapa_shared(BAR_SFREE(0), 0);

    if constexpr (C::ROLE == ROLE_DQ) {
      const uint16_t* Og = reinterpret_cast<const uint16_t*>(p.o) + b * p.o_sb + h * p.o_sh;
      const uint16_t* dOg = reinterpret_cast<const uint16_t*>(p.dout) + b * p.do_sb + h * p.do_sh;
      tile_delta<C::D, C::BF16, M>(Og, p.o_sn, dOg, p.do_sn, r0, N, rwi, 4 * RW, lane, sRow, p.delta + rowbase_q);
      asm volatile("bar.sync 1, %0;" ::"n"(128 * C::RW) : "memory");
      row_delta = sRow[row];
      row_lse2 = (r0 + row < N) ? p.lse[rowbase_q + r0 + row] * LOG2E : 0.f;
    }

    // Materialised backward (dQ role): workspace block of item 0 of this
    // (b, h, q tile); item i is block ws_blk0 + i, its dS block ws_blocks later.
    long long ws_blk0 = 0;
    if constexpr (C::ROLE == ROLE_DQ) {
      if (p.ws != nullptr)
        ws_blk0 = (static_cast<long long>(b) * p.Hq + h) * p.ws_bph + ws_blocks_before(tile, N, p.causal, p.window);
    }
    if constexpr (C::ROLE == ROLE_FWD) {
      // Online softmax (exp2 domain, lazy rescaling as in attn_kernel.cuh) over
      // the BN/2 columns of every item this thread holds. The two warps holding
      // the same 64 rows (quadrants q and q^2) exchange their maxima through
      // shared memory once per item, so both halves of a row share one running
      // max; each keeps a partial row sum, added in the epilogue. The exchange
      // barrier runs on every item even after a failed wait, so a partner warp
      // is never left at it.
      const int pbar = 2 + (q4 & 1);
      const int part = half * RW + cs;  // which part of the row's columns this warp holds
      auto pair_sync = [&]() { asm volatile("bar.sync %0, %1;" ::"r"(pbar), "n"(64 * C::RW) : "memory"); };
      float m_run = -INFINITY, l_run = 0.f;
      for (int i = 0; i < n_items; ++i) {
        const int sb = i % NS;
        const int cb = item_col0(i) + half * (BN / 2);
        const long long t_w = tick();
        if (ok) {
          ok = mbar_wait_cluster(BAR_SFULL(sb), (i / NS) & 1u, abort_flag, p.status, ST_TIMEOUT_SCORES, p.wait_limit);
          ok = __all_sync(0xffffffffu, ok);
        }
        tock(WC_ROW_SFULL, t_w);
        const long long t_work = tick();
        const uint32_t s_col = C::ACC_COLS + sb * C::SBUF_COLS;
        // Two passes over S in TMEM, 32 columns at a time with rolled loops:
        // the row max, then exp2 / sum / pack into the P buffer. Re-reading S
        // costs TMEM bandwidth, which is plentiful; unrolling both passes over
        // all columns would multiply the code size, and the instruction cache
        // is shared with the MMA-issuing thread.
        int lo_abs, hi_abs;
        attended_interval(true, r0 + row, N, p.Nk, p.qoff, p.causal, p.window, lo_abs, hi_abs);
        const int lo_rel = lo_abs - cb;
        const unsigned span = span_of(lo_rel, hi_abs - cb);
        float mx = -INFINITY;
        if (ok) {
          tc_fence_after();
#pragma unroll 1
          for (int kb = kc0; kb < kc0 + KCHW; kb += 2) {
            uint32_t rs[2][32];
            tmem_ld32_async(tq + s_col + 32 * kb, rs[0]);
            tmem_ld32_async(tq + s_col + 32 * (kb + 1), rs[1]);
            tmem_ld_wait32(rs[0]);
            tmem_ld_wait32(rs[1]);
#pragma unroll
            for (int u = 0; u < 2; ++u) {
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                const int c = 32 * (kb + u) + j;
                const float x = __uint_as_float(rs[u][j]);
                mx = (static_cast<unsigned>(c - lo_rel) < span) ? fmaxf(mx, x) : mx;
              }
            }
          }
          mx *= sl2;  // sl2 > 0, so the max commutes with the scaling
        }
        float* xm = sX + (i & 1) * 2 * RW * M;
        xm[part * M + row] = mx;
        pair_sync();
#pragma unroll
        for (int pt = 0; pt < 2 * RW; ++pt) mx = fmaxf(mx, xm[pt * M + row]);
        if (!ok) continue;
        float alpha = 1.f;
        bool rescale = false;
        const float m_new = fmaxf(m_run, mx);
        if (m_new > m_run + 8.f) {
          if (i > 0) {
            alpha = ex2(m_run - m_new);
            rescale = true;
          }
          m_run = m_new;
        }
        const float ms = (m_run == -INFINITY) ? 0.f : m_run;
        float sum = 0.f;
#pragma unroll 1
        for (int k = kc0; k < kc0 + KCHW; ++k) {
          uint32_t r[32];
          tmem_ld32(tq + s_col + 32 * k, r);
          float e[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int c = 32 * k + j;
            const float x = ex2(__uint_as_float(r[j]) * sl2 - ms);
            e[j] = (static_cast<unsigned>(c - lo_rel) < span) ? x : 0.f;
            sum += e[j];
          }
          // K-major SWIZZLE_128B [64 rows x BN] tile of 64-column panels.
          const int col = half * (BN / 2) + 32 * k;
          uint8_t* prow = sP + sb * C::PBUF_ONE + (col / 64) * (M * 128) + row * 128;
#pragma unroll
          for (int cc = 0; cc < 4; ++cc) {
            const int chunk16 = (col % 64) / 8 + cc;
            uint4 w;
            w.x = pack2<C::BF16>(e[8 * cc + 0], e[8 * cc + 1]);
            w.y = pack2<C::BF16>(e[8 * cc + 2], e[8 * cc + 3]);
            w.z = pack2<C::BF16>(e[8 * cc + 4], e[8 * cc + 5]);
            w.w = pack2<C::BF16>(e[8 * cc + 6], e[8 * cc + 7]);
            *reinterpret_cast<uint4*>(prow + ((chunk16 ^ (row & 7)) * 16)) = w;
          }
        }
        l_run = l_run * alpha + sum;
        if (__any_sync(0xffffffffu, rescale)) {
          // O's rows are rescaled in place once the previous item's P V
          // MMAs have landed (this thread's quadrant, all ACC_COLS columns).
          ok = mbar_wait_cluster(BAR_ACC, (i - 1) & 1u, abort_flag, p.status, ST_TIMEOUT_ACC, p.wait_limit);
          ok = __all_sync(0xffffffffu, ok);
          if (!ok) continue;
          tc_fence_after();
#pragma unroll 1
          for (int k = cs * (C::ACC_COLS / 32 / RW); k < (cs + 1) * (C::ACC_COLS / 32 / RW); k += 2) {
            uint32_t r[2][32];
            tmem_ld32_async(tq + 32 * k, r[0]);
            tmem_ld32_async(tq + 32 * (k + 1), r[1]);
            tmem_ld_wait32(r[0]);
            tmem_ld_wait32(r[1]);
#pragma unroll
            for (int u = 0; u < 2; ++u) {
#pragma unroll
              for (int j = 0; j < 32; ++j) r[u][j] = __float_as_uint(__uint_as_float(r[u][j]) * alpha);
              tmem_st32(tq + 32 * (k + u), r[u]);
            }
          }
          tmem_st_wait();
        }
        tc_fence_before();
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive_remote(pready_l0 + 8u * sb);
        tock(WC_ROW_WORK, t_work);
      }

      // ---------------- epilogue ----------------
      const long long t_epi = tick();
      float* xl = sX + 4 * RW * M;
      xl[part * M + row] = l_run;
      pair_sync();
      float l_tot = 0.f;
#pragma unroll
      for (int pt = 0; pt < 2 * RW; ++pt) l_tot += xl[pt * M + row];
      if (ok && n_items > 0) {
        ok = mbar_wait_cluster(BAR_FINAL, 0, abort_flag, p.status, ST_TIMEOUT_ACC, p.wait_limit);
        ok = __all_sync(0xffffffffu, ok);
      }
      if (ok && n_items > 0) {
        tc_fence_after();
        const float mul = (l_tot > 0.f) ? 1.f / l_tot : 0.f;
        const int orow = r0 + row;
        const long long obase = static_cast<long long>(b) * p.out_sb + static_cast<long long>(h) * p.out_sh +
                                static_cast<long long>(orow) * p.out_sn;
#pragma unroll 1
        for (int e = cs * (4 * C::NACC / RW); e < (cs + 1) * (4 * C::NACC / RW); ++e) {
          const int g = e >> 2, k = e & 3;
          {
            uint32_t r[32];
            tmem_ld32(tq + g * 128 + 32 * k, r);
            float v[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]) * mul;
            if (orow < N) store_row32<C::BF16>(p.out, obase + 256 * g + 128 * half + 32 * k, v);
          }
        }
        if (p.lse != nullptr && part == 0 && orow < N) {
          const float LN2 = 0.6931471805599453f;
          p.lse[rowbase_q + orow] = (l_tot > 0.f) ? (m_run + __log2f(l_tot)) * LN2 : -INFINITY;
        }
      }
      tock(WC_ROW_EPILOGUE, t_epi);
    } else {
      // Materialised backward (dQ role with a workspace): P and then dS of
      // every item pass through the P buffer, from which TMA stores them to
      // the workspace as one [64 rows x 256] block slice per CTA. The four row
      // warps synchronise on a named barrier around each store, so no warp
      // leaves the loop early: after a failed wait a warp skips its work but
      // still reaches every barrier.
      const bool ws_on = (C::ROLE == ROLE_DQ && BN == 256) && p.ws != nullptr;
      const bool tid0 = (warp == 4 && lane == 0);
      auto row_bar = [&]() { asm volatile("bar.sync 1, %0;" ::"n"(128 * C::RW) : "memory"); };
      // K-major SWIZZLE_128B [64 rows x BN] tile of 64-column panels.
      auto put = [&](int sb, int k, const float (&vals)[32]) {
        const int col = half * (BN / 2) + 32 * k;  // column within the item
        uint8_t* prow = sP + sb * C::PBUF_ONE + (col / 64) * (M * 128) + row * 128;
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
          const int chunk16 = (col % 64) / 8 + cc;
          uint4 w;
          w.x = pack2<C::BF16>(vals[8 * cc + 0], vals[8 * cc + 1]);
          w.y = pack2<C::BF16>(vals[8 * cc + 2], vals[8 * cc + 3]);
          w.z = pack2<C::BF16>(vals[8 * cc + 4], vals[8 * cc + 5]);
          w.w = pack2<C::BF16>(vals[8 * cc + 6], vals[8 * cc + 7]);
          *reinterpret_cast<uint4*>(prow + ((chunk16 ^ (row & 7)) * 16)) = w;
        }
      };
      // The workspace is read once, by the dK/dV kernel: store it evict-first.
      const uint64_t ws_pol = l2_policy_evict_first();
      auto store_block = [&](int sb, long long blk) {
#pragma unroll
        for (int c = 0; c < BN / 64; ++c)
          tma_store_3d_hint(&tmWS, smem_u32(sP + sb * C::PBUF_ONE + c * (M * 128)), 64 * c,
                            M * static_cast<int>(rank), static_cast<int>(blk), ws_pol);
        bulk_commit();
      };
      for (int i = 0; i < n_items; ++i) {
        const int sb = i % NS;
        const int c0 = item_col0(i);
        const int cb = c0 + half * (BN / 2);  // first column this thread owns
        // Per-column softmax statistics (DK / DV), fetched before waiting so the
        // global-load latency overlaps the MMAs.
        float col_lse2[KCHW], col_delta[KCHW];
        if constexpr (!C::ROWS_ARE_Q) {
          const int hq = item_headC(i);
          const long long colbase = (static_cast<long long>(b) * p.Hq + hq) * N;
#pragma unroll
          for (int k = 0; k < KCHW; ++k) {
            const int qq = cb + 32 * (kc0 + k) + lane;
            col_lse2[k] = (qq < N) ? p.lse[colbase + qq] * LOG2E : 0.f;
            col_delta[k] = (C::HAS_DP && qq < N) ? p.delta[colbase + qq] : 0.f;
          }
        }
        const long long t_w = tick();
        // dQ / dK: wait for S only; dP is waited for after P is computed.
        if (ok) {
          ok = mbar_wait_cluster(C::HAS_DP ? BAR_SREADY(sb) : BAR_SFULL(sb), (i / NS) & 1u, abort_flag, p.status,
                                 ST_TIMEOUT_SCORES, p.wait_limit);
          ok = __all_sync(0xffffffffu, ok);
        }
        tock(WC_ROW_SFULL, t_w);
        const long long t_work = tick();
        const uint32_t s_col = C::ACC_COLS + sb * C::SBUF_COLS;
        const uint32_t dp_col = C::ACC_COLS + (NS + sb) * C::SBUF_COLS;
        constexpr int KB = KCHW < 2 ? KCHW : 2;  // chunks loaded per TMEM round trip (register budget)
        // P = exp2(S * scale * log2 e - lse * log2 e), masked, for all columns this thread owns
        // (local chunk k is column chunk kc0 + k of the item).
        float pv[KCHW][32];
        if (ok) {
          tc_fence_after();
          int lo_abs, hi_abs;
          attended_interval(C::ROWS_ARE_Q, r0 + row, N, p.Nk, p.qoff, p.causal, p.window, lo_abs, hi_abs);
          const int lo_rel = lo_abs - cb;
          const unsigned span = span_of(lo_rel, hi_abs - cb);
#pragma unroll
          for (int kb = 0; kb < KCHW; kb += KB) {
            uint32_t rs[KB][32];
#pragma unroll
            for (int u = 0; u < KB; ++u) tmem_ld32_async(tq + s_col + 32 * (kc0 + kb + u), rs[u]);
#pragma unroll
            for (int u = 0; u < KB; ++u) tmem_ld_wait32(rs[u]);
#pragma unroll
            for (int u = 0; u < KB; ++u) {
              const int k = kb + u;
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                const float l2 = C::ROWS_ARE_Q ? row_lse2 : __shfl_sync(0xffffffffu, col_lse2[k], j);
                const float e = ex2(__uint_as_float(rs[u][j]) * sl2 - l2);
                pv[k][j] = (static_cast<unsigned>(32 * (kc0 + k) + j - lo_rel) < span) ? e : 0.f;
              }
            }
          }
        }
        if constexpr (C::EARLY_S) {
          if (ok) {  // S is in registers: the issuer may overwrite it
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_remote(sfree_l0);
          }
        }
        if (ws_on) {
          // P -> buffer -> workspace. The buffer still holds dS of the previous
          // item: wait for its accumulate MMAs (with EARLY_S, S-ready no longer
          // implies them) and for its TMA store to have read it.
          if (C::EARLY_S && i > 0 && ok) {
            ok = mbar_wait_cluster(BAR_ACC, (i - 1) & 1u, abort_flag, p.status, ST_TIMEOUT_ACC, p.wait_limit);
            ok = __all_sync(0xffffffffu, ok);
          }
          if (tid0) bulk_wait_read0();
          row_bar();
          if (ok) {
#pragma unroll
            for (int k = 0; k < KCHW; ++k) put(sb, kc0 + k, pv[k]);
            fence_proxy_async_smem();
          }
          row_bar();
          if (tid0 && ok) store_block(sb, ws_blk0 + i);
        }
        if (C::HAS_DP && ok) {
          ok = mbar_wait_cluster(BAR_SFULL(sb), (i / NS) & 1u, abort_flag, p.status, ST_TIMEOUT_SCORES, p.wait_limit);
          ok = __all_sync(0xffffffffu, ok);
          if (ok) tc_fence_after();
        }
        if (ws_on) {
          if (tid0) bulk_wait_read0();  // the P store has read the buffer
          row_bar();
        }
        if (ok) {
#pragma unroll
          for (int kb = 0; kb < KCHW; kb += KB) {
            uint32_t rd[KB][32];
            if constexpr (C::HAS_DP) {
#pragma unroll
              for (int u = 0; u < KB; ++u) tmem_ld32_async(tq + dp_col + 32 * (kc0 + kb + u), rd[u]);
#pragma unroll
              for (int u = 0; u < KB; ++u) tmem_ld_wait32(rd[u]);
            }
#pragma unroll
            for (int u = 0; u < KB; ++u) {
              const int k = kb + u;
              float v[32];
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                if constexpr (C::HAS_DP) {
                  const float dl = C::ROWS_ARE_Q ? row_delta : __shfl_sync(0xffffffffu, col_delta[k], j);
                  v[j] = pv[k][j] * (__uint_as_float(rd[u][j]) - dl);
                } else {
                  v[j] = pv[k][j];
                }
              }
              put(sb, kc0 + k, v);
            }
          }
          tc_fence_before();
          fence_proxy_async_smem();
        }
        if (ws_on) {
          row_bar();
          if (tid0 && ok) store_block(sb, p.ws_blocks + ws_blk0 + i);
        }
        if (ok) {
          __syncwarp();
          if (lane == 0) mbar_arrive_remote(pready_l0 + 8u * sb);
        }
        tock(WC_ROW_WORK, t_work);
      }
      if (ws_on && tid0) bulk_wait0();  // workspace writes complete before the CTA exits

      // ---------------- epilogue ----------------
      const long long t_epi = tick();
      if (ok && n_items > 0) {
        ok = mbar_wait_cluster(BAR_FINAL, 0, abort_flag, p.status, ST_TIMEOUT_ACC, p.wait_limit);
        ok = __all_sync(0xffffffffu, ok);
      }
      if (ok && n_items > 0) {
        tc_fence_after();
        const float mul = (C::ROLE == ROLE_DV) ? 1.f : p.scale;
        const int orow = r0 + row;
        const long long obase = static_cast<long long>(b) * p.out_sb + static_cast<long long>(h) * p.out_sh +
                                static_cast<long long>(orow) * p.out_sn;
#pragma unroll 1
        for (int e = cs * (4 * C::NACC / RW); e < (cs + 1) * (4 * C::NACC / RW); ++e) {
          const int g = e >> 2, k = e & 3;
          {
            uint32_t r[32];
            tmem_ld32(tq + g * 128 + 32 * k, r);
            float v[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]) * mul;
            if (orow < N)
              store_out32<C::BF16>(p.out, obase + 256 * g + 128 * half + 32 * k, v, !C::ROWS_ARE_Q && p.out_f32);
          }
        }
      }
      tock(WC_ROW_EPILOGUE, t_epi);
    }
  }

  if (prof) {
    // one reporter per role: producer lane 0, MMA lane 0 (leader), warp 4 lane 0, thread 0
    const bool reporter = (lane == 0 && (warp == 0 || warp == 1 || warp == 4));
    if (reporter) {
      for (int k = 0; k < WC_CTA_TOTAL; ++k)
        if (wc[k]) atomicAdd(p.prof + k, wc[k]);
    }
    if (threadIdx.x == 0) {
      atomicAdd(p.prof + WC_CTA_TOTAL, static_cast<unsigned long long>(clock64() - t_start));
      atomicAdd(p.prof + WC_CTAS, 1ULL);
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // the peer has finished reading this CTA's TMEM / smem and arriving on its barriers
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tbase, 512);
  }
}

}  // namespace gqafa
