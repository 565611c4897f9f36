// One warp-specialised tcgen05 kernel template that covers the four launches of
// the GQA flash-attention path:
//
//   ROLE_FWD : O   = softmax(scale * Q K^T + mask) V           (+ LSE)
//              reference: _flash_attn_gqa_kernel, flash_attn/attention.py:244-388
//   ROLE_DQ  : dQ  = scale * sum_j dS_j K_j, dS = P o (dO V^T - delta)
//              with delta = rowsum(dO o O) computed in the prologue
//              reference: _flash_attn_gqa_bwd_dq_kernel (STORE_DELTA=True),
//              flash_attn/attention.py:686-797
//   ROLE_DK  : dK  = scale * sum over the G query heads and q blocks of dS^T Q
//   ROLE_DV  : dV  = sum over the G query heads and q blocks of P^T dO
//              reference (both): _flash_attn_gqa_bwd_dkv_packed_kernel,
//              flash_attn/attention.py:1079-1213 (packed GQA: one program per KV
//              block loops over every Q head of its group, no atomics)
//
// This 1-CTA template runs head_dim 64, 128 and 256 (the whole fp32
// accumulator of a 128-row tile plus the score buffers fit one SM's 512 TMEM
// columns); head_dim 512 runs on CTA pairs (attn_pair_kernel.cuh).
//
// Structure of one CTA (256 threads):
//   warp 0      TMA producer: loads the resident row tile (R1, R2) once, then
//               streams 64-column panels of the column operands through a ring.
//   warp 1      allocates TMEM and issues every tcgen05.mma from one thread.
//   warps 4..7  "row" warps (warp w reads TMEM lane quadrant w % 4): read
//               scores from TMEM, apply mask / softmax / gradient algebra,
//               write P or dS (16-bit) back into the score columns, run the
//               epilogue.
//
// A "row tile" is 128 rows that stay resident (Q rows for FWD/DQ, K rows for
// DK/DV). The kernel loops over "items": column blocks of BN rows of the other
// operand (KV blocks for FWD/DQ; (query head, Q block) pairs for DK/DV).
// Per item:
//   scores  S  = R1 . C1^T              (K-major x K-major, contraction over D)
//           dP = R2 . C2^T              (DQ / DK only)
//   acc    += X . Y                     (X = P or dS read from TMEM, Y streamed
//                                        MN-major, contraction over BN)
//
// Tensor-memory layout: the accumulator in columns [0, D), the score buffers
// (S, and dP for DQ / DK) after it; lane = row of the tile.
#pragma once
#include "ptx_sm100.cuh"

namespace gqafa {

enum Role : int { ROLE_FWD = 0, ROLE_DQ = 1, ROLE_DK = 2, ROLE_DV = 3 };

struct KParams {
  int B, Hq, Hkv, N, G;
  // Key length and the query rows' offset into it: query row r sits at key
  // position r + qoff (qoff = Nk - N, the last N positions of a KV cache).
  // The backward runs with Nk == N and qoff == 0.
  int Nk, qoff;
  int causal, window;  // window > 0 only meaningful with causal (reference semantics)
  float scale, scale_log2;
  int num_row_tiles;  // row tiles in this launch
  int tile_begin;     // first row tile (row-range launches; 0 otherwise)
  int row_begin, row_end;  // host-side: rows this launch covers
  void* out;  // O / dQ / dK / dV, element strides below (last dim contiguous)
  long long out_sb, out_sh, out_sn;
  float* lse;    // [B, Hq, N] fp32, natural log, includes the softmax scale
  float* delta;  // [B, Hq, N] fp32
  const void* o;
  long long o_sb, o_sh, o_sn;
  const void* dout;
  long long do_sb, do_sh, do_sn;
  int* status;
  // Materialised backward (head_dim 512): the dQ kernel also writes P and dS
  // into `ws` when it is non-null; the dK/dV kernel reads them back and
  // writes dK to `out` and dV to `out2`. Layout: ws_blocks blocks of P, then
  // ws_blocks blocks of dS; block (b, h, q tile t, key block j) holds
  // [128 queries][256 keys] 16-bit values, row-major, at index
  // (b * Hq + h) * ws_bph + ws_blocks_before(t) + (j - first key block of t).
  void* ws;
  long long ws_bph, ws_blocks;
  void* out2;
  long long out2_sb, out2_sh, out2_sn;
  // Optional diagnostics: when non-null, each CTA adds the cycles its roles
  // spend waiting (see WaitCounter) into these counters. Null on the hot path.
  unsigned long long* prof;
  // Bound of every mbarrier wait, in clock cycles (WAIT_LIMIT_CYCLES unless a
  // test set a short one), and a test switch that makes the TMA producer
  // issue nothing, so every wait of the launch runs into that bound.
  long long wait_limit;
  int no_loads;
  // dK / dV outputs (out, out2 of the DK, DV and dK+dV roles) are fp32 rather
  // than the input dtype: partial sums that a caller adds up before rounding.
  int out_f32;
};

// Indices of the wait-cycle diagnostics counters.
enum WaitCounter : int {
  WC_PRODUCER_EMPTY = 0,  // producer waiting for a free ring stage
  WC_MMA_FULL_SCORES = 1, // MMA issuer waiting for score operands to land
  WC_MMA_FULL_Y = 2,      // MMA issuer waiting for accumulate operands to land
  WC_MMA_PREADY = 3,      // MMA issuer waiting for the row warps' P / dS
  WC_ROW_SFULL = 4,       // row warp (lane 0 of warp 4) waiting for scores
  WC_ROW_WORK = 5,        // row warp elementwise work per item
  WC_ROW_EPILOGUE = 6,    // row warp waiting for the final MMA + storing
  WC_CTA_TOTAL = 7,       // whole CTA lifetime (thread 0)
  WC_CTAS = 8,            // number of CTAs that reported
  WC_NUM = 9
};

// Key blocks (256 keys each) that query tile t (rows 128t .. 128t+127)
// attends: [jlo, jlo + jn). Same ranges as the head_dim-512 dQ kernel's items.
__host__ __device__ __forceinline__ void ws_key_blocks(int t, int N, int causal, int window, int& jlo, int& jn) {
  const int kv_hi = causal ? min(N, 128 * t + 128) : N;
  const int kv_lo = (causal && window > 0) ? max(0, 128 * t - window + 1) : 0;
  jlo = kv_lo / 256;
  jn = (kv_hi + 255) / 256 - jlo;
}

// Blocks stored for query tiles 0 .. t-1 of one head (t <= number of tiles).
__host__ __device__ inline long long ws_blocks_before(int t, int N, int causal, int window) {
  const int T = (N + 127) / 128;
  if (!causal) return static_cast<long long>(t) * ((N + 255) / 256);
  if (window == 0 && t <= T - 1) {
    // tiles t' < t <= T-1 end before N: tile t' has ceil((t'+1)/2) blocks
    const long long h = t / 2;
    return (t % 2 == 0) ? h * (h + 1) : (h + 1) * (h + 1);
  }
  long long n = 0;
  for (int u = 0; u < t; ++u) {
    int jlo, jn;
    ws_key_blocks(u, N, causal, window, jlo, jn);
    n += jn;
  }
  return n;
}

template <int ROLE_, int D_, int BN_, int NS_, int NSTAGES_, int YGROUP_, bool BF16_>
struct Cfg {
  static constexpr int ROLE = ROLE_, M = 128, D = D_, BN = BN_, NS = NS_;
  static constexpr int NSTAGES = NSTAGES_, YGROUP = YGROUP_;
  static constexpr bool BF16 = BF16_;
  static constexpr bool PAIR = false;
  static constexpr int MP = M;  // rows of one grid tile
  static constexpr bool HAS_DP = (ROLE == ROLE_DQ || ROLE == ROLE_DK);
  static constexpr bool ROWS_ARE_Q = (ROLE == ROLE_FWD || ROLE == ROLE_DQ);
  static constexpr int NCHUNK = 1;
  static constexpr int PANELS_D = D / 64;
  static constexpr int PANELS_Y = D / 64;
  static constexpr int R_PANEL = M * 128;
  static constexpr int STAGE_BYTES = BN * 128;
  static constexpr int C_BOX = BN, Y_BOX = BN;  // TMA box rows of the streamed operands
  static constexpr int R_BYTES = PANELS_D * R_PANEL * (HAS_DP ? 2 : 1);
  static constexpr int RING_BYTES = NSTAGES * STAGE_BYTES;
  static constexpr int NBARS = 2 * NSTAGES + 1 + 2 * NS + 2;
  static constexpr int MISC_BYTES = M * 4 + NBARS * 8 + 16;
  static constexpr int SMEM_BYTES = 1024 + R_BYTES + RING_BYTES + MISC_BYTES;
  // TMEM columns: accumulator [0, D), score buffers from S_COL0
  static constexpr int S_COL0 = D;
  static constexpr int SCORE_COLS = NS * BN * (HAS_DP ? 2 : 1);
  static constexpr uint32_t IDESC_S = make_idesc(M, BN, BF16, false);
  static constexpr uint32_t IDESC_Y = make_idesc(M, 64 * YGROUP, BF16, true);

  static_assert(D % 64 == 0 && D <= 256, "D");
  static_assert(BN % 32 == 0 && BN >= 32 && BN <= 256 && BN % 16 == 0, "BN");
  static_assert(D + SCORE_COLS <= 512, "TMEM");
  static_assert(PANELS_D % YGROUP == 0 && NSTAGES % YGROUP == 0, "ring groups");
  static_assert(SMEM_BYTES <= 232448, "shared memory");
};

// The columns a row attends form one interval [lo, hi) of absolute indices:
// for a query row q at key position q' = q + qoff, keys max(0, q'-W+1) .. q'
// (causal) or 0 .. Nk-1; for a key row k (backward, Nk == N), queries
// k .. min(k+W-1, N-1) (causal) or 0 .. N-1. Masking is then one unsigned
// compare per element (an element test inside the unrolled loops costs far
// more).
__device__ __forceinline__ void attended_interval(bool row_is_query, int row, int N, int Nk, int qoff, int causal,
                                                  int window, int& lo, int& hi) {
  if (row >= N) {
    lo = 0;
    hi = 0;
    return;
  }
  if (!causal) {
    lo = 0;
    hi = row_is_query ? Nk : N;
  } else if (row_is_query) {
    lo = window > 0 ? max(0, row + qoff - window + 1) : 0;
    hi = row + qoff + 1;
  } else {
    lo = row;
    hi = window > 0 ? min(N, row + window) : N;
  }
}

// Number of in-range columns for relative index test: keep iff
// (unsigned)(c - lo_rel) < span.
__device__ __forceinline__ unsigned span_of(int lo_rel, int hi_rel) {
  return hi_rel > lo_rel ? static_cast<unsigned>(hi_rel - lo_rel) : 0u;
}

// This lane's part of dot(a, b) over one row of D 16-bit values: 16-byte
// loads for D >= 256 (8 values per lane per pass), 8-byte loads at D = 128 and
// 4-byte loads at D = 64, so the warp reads the row in coalesced passes. The
// caller reduces over the warp.
template <int D, bool BF16>
__device__ __forceinline__ float row_dot(const uint16_t* a, const uint16_t* b, int lane) {
  float acc = 0.f;
  if constexpr (D >= 256) {
#pragma unroll
    for (int it = 0; it < D / 256; ++it) {
      const uint4 x = __ldg(reinterpret_cast<const uint4*>(a + it * 256 + lane * 8));
      const uint4 y = __ldg(reinterpret_cast<const uint4*>(b + it * 256 + lane * 8));
      const uint32_t xw[4] = {x.x, x.y, x.z, x.w}, yw[4] = {y.x, y.y, y.z, y.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        acc += unpack_lo<BF16>(xw[e]) * unpack_lo<BF16>(yw[e]);
        acc += unpack_hi<BF16>(xw[e]) * unpack_hi<BF16>(yw[e]);
      }
    }
  } else if constexpr (D == 128) {
    const uint2 x = __ldg(reinterpret_cast<const uint2*>(a + lane * 4));
    const uint2 y = __ldg(reinterpret_cast<const uint2*>(b + lane * 4));
    const uint32_t xw[2] = {x.x, x.y}, yw[2] = {y.x, y.y};
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      acc += unpack_lo<BF16>(xw[e]) * unpack_lo<BF16>(yw[e]);
      acc += unpack_hi<BF16>(xw[e]) * unpack_hi<BF16>(yw[e]);
    }
  } else {
    static_assert(D == 64, "head_dim");
    const uint32_t xw = __ldg(reinterpret_cast<const unsigned int*>(a + lane * 2));
    const uint32_t yw = __ldg(reinterpret_cast<const unsigned int*>(b + lane * 2));
    acc += unpack_lo<BF16>(xw) * unpack_lo<BF16>(yw);
    acc += unpack_hi<BF16>(xw) * unpack_hi<BF16>(yw);
  }
  return acc;
}

// delta = rowsum(dO o O) for rows r_first, r_first + r_step, ... < M of the
// tile starting at query row r0 (reference: the STORE_DELTA prologue,
// flash_attn/attention.py:733-742), one warp per row. The loads of RB rows
// are issued before any of their reductions, so their memory latencies
// overlap instead of adding up. Writes sRow[r] and delta[r0 + r] (rows < N).
template <int D, bool BF16, int M>
__device__ __forceinline__ void tile_delta(const uint16_t* Og, long long o_sn, const uint16_t* dOg, long long do_sn,
                                           int r0, int N, int r_first, int r_step, int lane, float* sRow,
                                           float* delta) {
  constexpr int RB = (D >= 512) ? 2 : 4;
  for (int r = r_first; r < M; r += RB * r_step) {
    float acc[RB];
#pragma unroll
    for (int u = 0; u < RB; ++u) {
      const int rr = r + u * r_step, q = r0 + rr;
      acc[u] = (rr < M && q < N) ? row_dot<D, BF16>(Og + q * o_sn, dOg + q * do_sn, lane) : 0.f;
    }
#pragma unroll
    for (int u = 0; u < RB; ++u) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc[u] += __shfl_xor_sync(0xffffffffu, acc[u], o);
      const int rr = r + u * r_step, q = r0 + rr;
      if (lane == 0 && rr < M) {
        sRow[rr] = acc[u];
        if (q < N) delta[q] = acc[u];
      }
    }
  }
}

template <bool BF16>
__device__ __forceinline__ void store_row32(void* base, long long off_elems, const float (&v)[32]);

// 32 values of an output row: 16-bit like the inputs, or fp32 when f32.
template <bool BF16>
__device__ __forceinline__ void store_out32(void* base, long long off_elems, const float (&v)[32], bool f32) {
  if (f32) {
    float4* dst = reinterpret_cast<float4*>(reinterpret_cast<float*>(base) + off_elems);
#pragma unroll
    for (int i = 0; i < 8; ++i) dst[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
  } else {
    store_row32<BF16>(base, off_elems, v);
  }
}

template <bool BF16>
__device__ __forceinline__ void store_row32(void* base, long long off_elems, const float (&v)[32]) {
  uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(base) + off_elems);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint4 w;
    w.x = pack2<BF16>(v[8 * i + 0], v[8 * i + 1]);
    w.y = pack2<BF16>(v[8 * i + 2], v[8 * i + 3]);
    w.z = pack2<BF16>(v[8 * i + 4], v[8 * i + 5]);
    w.w = pack2<BF16>(v[8 * i + 6], v[8 * i + 7]);
    dst[i] = w;
  }
}

template <class C>
__global__ void __launch_bounds__(256, 1)
    attn_kernel(const __grid_constant__ CUtensorMap tmR1, const __grid_constant__ CUtensorMap tmR2,
                const __grid_constant__ CUtensorMap tmC1, const __grid_constant__ CUtensorMap tmC2,
                const __grid_constant__ CUtensorMap tmY, const KParams p) {
  constexpr int M = C::M, BN = C::BN, NS = C::NS, NST = C::NSTAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sR1 = smem;
  uint8_t* sR2 = smem + C::PANELS_D * C::R_PANEL;
  uint8_t* sRing = smem + C::R_BYTES;
  float* sRow = reinterpret_cast<float*>(sRing + C::RING_BYTES);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sRow + M);
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

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  // ---- tile decode: heads fastest so the query heads of one KV group run together
  const int heads = C::ROWS_ARE_Q ? p.Hq : p.Hkv;
  int idx = blockIdx.x;
  const int h = idx % heads;
  idx /= heads;
  const int b = idx % p.B;
  idx /= p.B;
  // FWD/DQ: the last q tiles carry the most causal work, launch them first.
  const int tile = p.tile_begin + (C::ROWS_ARE_Q ? (p.num_row_tiles - 1 - idx) : idx);
  const int r0 = tile * M;
  const int N = p.N, G = p.G;
  const bool swa = p.causal && p.window > 0;

  int jlo, jn, n_items;
  if constexpr (C::ROWS_ARE_Q) {
    const int kv_hi = p.causal ? min(p.Nk, r0 + M + p.qoff) : p.Nk;
    const int kv_lo = swa ? max(0, r0 + p.qoff - p.window + 1) : 0;
    jlo = kv_lo / BN;
    jn = (kv_hi + BN - 1) / BN - jlo;
    n_items = jn;
  } else {
    const int q_lo = p.causal ? r0 : 0;
    const int q_hi = swa ? min(N, r0 + M - 1 + p.window) : N;
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
      mbar_init(BAR_PREADY(s), 4);
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
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;

  if (warp == 0) {
    // ======================= TMA producer =======================
    if (lane == 0 && !p.no_loads) {
      bool ok = true;
      mbar_arrive_expect_tx(BAR_RFULL, C::R_BYTES);
      for (int pn = 0; pn < C::PANELS_D; ++pn)
        tma_load_4d(smem_u32(sR1 + pn * C::R_PANEL), &tmR1, BAR_RFULL, 64 * pn, r0, h, b);
      if constexpr (C::HAS_DP) {
        for (int pn = 0; pn < C::PANELS_D; ++pn)
          tma_load_4d(smem_u32(sR2 + pn * C::R_PANEL), &tmR2, BAR_RFULL, 64 * pn, r0, h, b);
      }
      uint32_t cnt = 0;
      auto load_panel = [&](const CUtensorMap* m, int x, int y, int hh) -> bool {
        const int st = cnt % NST;
        const uint32_t ph = (cnt / NST) & 1u;
        if (!mbar_wait(BAR_EMPTY(st), ph ^ 1u, abort_flag, p.status, ST_TIMEOUT_RING_EMPTY, p.wait_limit)) return false;
        mbar_arrive_expect_tx(BAR_FULL(st), C::STAGE_BYTES);
        tma_load_4d(smem_u32(sRing + st * C::STAGE_BYTES), m, BAR_FULL(st), x, y, hh, b);
        ++cnt;
        return true;
      };
      auto load_scores = [&](int i) -> bool {
        const int c0 = item_col0(i), hc = item_headC(i);
        for (int pn = 0; pn < C::PANELS_D; ++pn)
          if (!load_panel(&tmC1, 64 * pn, c0, hc)) return false;
        if constexpr (C::HAS_DP) {
          for (int pn = 0; pn < C::PANELS_D; ++pn)
            if (!load_panel(&tmC2, 64 * pn, c0, hc)) return false;
        }
        return true;
      };
      auto load_y = [&](int i) -> bool {
        const int c0 = item_col0(i), hc = item_headC(i);
        for (int pn = 0; pn < C::PANELS_Y; ++pn)
          if (!load_panel(&tmY, 64 * pn, c0, hc)) return false;
        return true;
      };
      for (int s = 0; s < NS && s < n_items && ok; ++s) ok = load_scores(s);
      for (int i = 0; i < n_items && ok; ++i) {
        ok = load_y(i);
        if (ok && i + NS < n_items) ok = load_scores(i + NS);
      }
    }
  } else if (warp == 1) {
    // ======================= MMA issuer =======================
    if (lane == 0) {
      bool ok = mbar_wait(BAR_RFULL, 0, abort_flag, p.status, ST_TIMEOUT_RESIDENT, p.wait_limit);
      tc_fence_after();
      const uint32_t aR1 = smem_u32(sR1), aR2 = smem_u32(sR2), aRing = smem_u32(sRing);
      uint32_t cnt = 0;
      auto scores_from = [&](uint32_t aR, uint32_t d_tmem) -> bool {
        for (int pn = 0; pn < C::PANELS_D; ++pn) {
          const int st = cnt % NST;
          if (!mbar_wait(BAR_FULL(st), (cnt / NST) & 1u, abort_flag, p.status, ST_TIMEOUT_RING_FULL, p.wait_limit))
            return false;
          tc_fence_after();
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint64_t ad = sw128_desc(aR + pn * C::R_PANEL + 32 * k, 16, 1024);
            const uint64_t bd = sw128_desc(aRing + st * C::STAGE_BYTES + 32 * k, 16, 1024);
            mma_ss(d_tmem, ad, bd, C::IDESC_S, (pn | k) != 0);
          }
          mma_commit(BAR_EMPTY(st));
          ++cnt;
        }
        return true;
      };
      auto issue_scores = [&](int i) -> bool {
        const int sb = i % NS;
        if (!scores_from(aR1, tbase + C::S_COL0 + sb * BN)) return false;
        if constexpr (C::HAS_DP) {
          if (!scores_from(aR2, tbase + C::S_COL0 + (NS + sb) * BN)) return false;
        }
        mma_commit(BAR_SFULL(sb));
        return true;
      };
      auto issue_acc = [&](int i) -> bool {
        const int sb = i % NS;
        if (!mbar_wait(BAR_PREADY(sb), (i / NS) & 1u, abort_flag, p.status, ST_TIMEOUT_PREADY, p.wait_limit)) return false;
        for (int j = 0; j < C::PANELS_Y; ++j) {
          const int st = (cnt + j) % NST;
          if (!mbar_wait(BAR_FULL(st), ((cnt + j) / NST) & 1u, abort_flag, p.status, ST_TIMEOUT_RING_FULL, p.wait_limit))
            return false;
        }
        tc_fence_after();
#pragma unroll 1
        for (int t = 0; t < BN / 16; ++t) {
#pragma unroll
          for (int g = 0; g < C::PANELS_Y / C::YGROUP; ++g) {
            const int st0 = (cnt + g * C::YGROUP) % NST;
            const uint64_t bd = sw128_desc(aRing + st0 * C::STAGE_BYTES + t * 2048, C::STAGE_BYTES, 1024);
            const uint32_t d_tmem = tbase + g * 64 * C::YGROUP;
            const uint32_t accum = (i > 0 || t > 0) ? 1u : 0u;
            mma_ts(d_tmem, tbase + C::S_COL0 + sb * BN + t * 8, bd, C::IDESC_Y, accum);
          }
        }
        mma_commit(BAR_ACC);
        for (int j = 0; j < C::PANELS_Y; ++j) mma_commit(BAR_EMPTY((cnt + j) % NST));
        cnt += C::PANELS_Y;
        return true;
      };
      for (int s = 0; s < NS && s < n_items && ok; ++s) ok = issue_scores(s);
      for (int i = 0; i < n_items && ok; ++i) {
        ok = issue_acc(i);
        if (ok && i + NS < n_items) ok = issue_scores(i + NS);
      }
      if (ok) mma_commit(BAR_FINAL);
    }
  } else if (warp >= 4) {
    // ======================= row warps =======================
    const int q4 = warp & 3;  // TMEM lane quadrant this warp may access
    const uint32_t tq = tbase + (static_cast<uint32_t>(q4 * 32) << 16);
    // Row owned by this thread in the score buffers and in the accumulator.
    const int srow = q4 * 32 + lane;  // row of the tile this thread owns (= its TMEM lane)
    const float LOG2E = 1.4426950408889634f;
    const float sl2 = p.scale_log2;
    bool ok = true;

    // per-row state
    float m_run = -INFINITY, l_run = 0.f;      // FWD
    float row_lse2 = 0.f, row_delta = 0.f;     // DQ
    const long long rowbase_q = (static_cast<long long>(b) * p.Hq + (C::ROWS_ARE_Q ? h : 0)) * N;

    if constexpr (C::ROLE == ROLE_DQ) {
      // delta = rowsum(dO o O), one warp per row, coalesced 16-byte loads.
      const uint16_t* Og = reinterpret_cast<const uint16_t*>(p.o) + b * p.o_sb + h * p.o_sh;
      const uint16_t* dOg = reinterpret_cast<const uint16_t*>(p.dout) + b * p.do_sb + h * p.do_sh;
      tile_delta<C::D, C::BF16, M>(Og, p.o_sn, dOg, p.do_sn, r0, N, q4, 4, lane, sRow, p.delta + rowbase_q);
      asm volatile("bar.sync 1, 128;" ::: "memory");
      row_delta = sRow[srow];
      row_lse2 = (r0 + srow < N) ? p.lse[rowbase_q + r0 + srow] * LOG2E : 0.f;
    }

    for (int i = 0; i < n_items && ok; ++i) {
      const int sb = i % NS;
      ok = mbar_wait(BAR_SFULL(sb), (i / NS) & 1u, abort_flag, p.status, ST_TIMEOUT_SCORES, p.wait_limit);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      const int c0 = item_col0(i);
      const uint32_t s_col = C::S_COL0 + sb * BN;
      const uint32_t dp_col = C::S_COL0 + (NS + sb) * BN;
      bool need_mask;
      if constexpr (C::ROWS_ARE_Q) {
        need_mask = (c0 + BN > p.Nk) || (p.causal && c0 + BN - 1 > r0 + p.qoff) ||
                    (swa && r0 + p.qoff + M - 1 - c0 >= p.window);
      } else {
        need_mask = (c0 + BN > N) || (p.causal && r0 + M - 1 > c0) ||
                    (swa && c0 + BN - 1 - r0 >= p.window);
      }
      int lo_abs, hi_abs;
      attended_interval(C::ROWS_ARE_Q, r0 + srow, N, p.Nk, p.qoff, p.causal, p.window, lo_abs, hi_abs);
      const int lo_rel = lo_abs - c0;
      const unsigned span = span_of(lo_rel, hi_abs - c0);
      auto valid = [&](int c) { return static_cast<unsigned>(c - lo_rel) < span; };

      if constexpr (C::ROLE == ROLE_FWD) {
        float s[BN];
#pragma unroll
        for (int k = 0; k < BN / 32; ++k) {
          uint32_t r[32];
          tmem_ld32(tq + s_col + 32 * k, r);
#pragma unroll
          for (int j = 0; j < 32; ++j) s[32 * k + j] = __uint_as_float(r[j]) * sl2;
        }
        float mx = -INFINITY;
        if (need_mask) {
#pragma unroll
          for (int c = 0; c < BN; ++c) {
            if (!valid(c)) s[c] = -INFINITY;
            mx = fmaxf(mx, s[c]);
          }
        } else {
#pragma unroll
          for (int c = 0; c < BN; ++c) mx = fmaxf(mx, s[c]);
        }
        // Lazy rescaling: keep the running max unless it grows by more than
        // 2^8; P then stays <= 256, which fp32 and 16-bit P represent with the
        // same relative precision. O and l always use the same max, so the
        // final O = acc / l is exact algebra.
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
#pragma unroll
        for (int c = 0; c < BN; ++c) {
          s[c] = ex2(s[c] - ms);
          sum += s[c];
        }
        l_run = l_run * alpha + sum;
        if (__any_sync(0xffffffffu, rescale)) {
          ok = mbar_wait(BAR_ACC, (i - 1) & 1u, abort_flag, p.status, ST_TIMEOUT_ACC, p.wait_limit);
          ok = __all_sync(0xffffffffu, ok);
          if (!ok) break;
          tc_fence_after();
#pragma unroll 1
          for (int k = 0; k < C::D / 32; ++k) {
            uint32_t r[32];
            tmem_ld32(tq + 32 * k, r);
#pragma unroll
            for (int j = 0; j < 32; ++j) r[j] = __float_as_uint(__uint_as_float(r[j]) * alpha);
            tmem_st32(tq + 32 * k, r);
          }
        }
#pragma unroll
        for (int k = 0; k < BN / 64; ++k) {
          uint32_t w[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) w[j] = pack2<C::BF16>(s[64 * k + 2 * j], s[64 * k + 2 * j + 1]);
          tmem_st32(tq + s_col + 32 * k, w);
        }
        if constexpr (BN % 64 != 0) {
          uint32_t w[16];
#pragma unroll
          for (int j = 0; j < 16; ++j)
            w[j] = pack2<C::BF16>(s[BN - 32 + 2 * j], s[BN - 32 + 2 * j + 1]);
          tmem_st16(tq + s_col + (BN - 32) / 2, w);
        }
      } else {
        // DQ / DK / DV: process 32 columns at a time.
        const int hq = C::ROWS_ARE_Q ? h : item_headC(i);
        const long long colbase = (static_cast<long long>(b) * p.Hq + hq) * N;
#pragma unroll 1
        for (int k = 0; k < BN / 32; ++k) {
          uint32_t rs[32];
          tmem_ld32(tq + s_col + 32 * k, rs);
          uint32_t rd[32];
          if constexpr (C::HAS_DP) tmem_ld32(tq + dp_col + 32 * k, rd);
          float col_lse2 = 0.f, col_delta = 0.f;
          if constexpr (!C::ROWS_ARE_Q) {
            const int qq = c0 + 32 * k + lane;
            if (qq < N) {
              col_lse2 = p.lse[colbase + qq] * LOG2E;
              if constexpr (C::HAS_DP) col_delta = p.delta[colbase + qq];
            }
          }
          float v[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            float l2, dl;
            if constexpr (C::ROWS_ARE_Q) {
              l2 = row_lse2;
              dl = row_delta;
            } else {
              l2 = __shfl_sync(0xffffffffu, col_lse2, j);
              dl = C::HAS_DP ? __shfl_sync(0xffffffffu, col_delta, j) : 0.f;
            }
            float pv = ex2(__uint_as_float(rs[j]) * sl2 - l2);
            pv = valid(32 * k + j) ? pv : 0.f;
            if constexpr (C::HAS_DP) {
              v[j] = pv * (__uint_as_float(rd[j]) - dl);
            } else {
              v[j] = pv;
            }
          }
          // P / dS as 16-bit pairs over the first half of this chunk's
          // score columns (the MMA reads A from TMEM)
          uint32_t w[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) w[j] = pack2<C::BF16>(v[2 * j], v[2 * j + 1]);
          tmem_st16(tq + s_col + 16 * k, w);
        }
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(BAR_PREADY(sb));
    }

    // ---------------- epilogue ----------------
    if (ok && n_items > 0) {
      ok = mbar_wait(BAR_FINAL, 0, abort_flag, p.status, ST_TIMEOUT_ACC, p.wait_limit);
      ok = __all_sync(0xffffffffu, ok);
    }
    if (ok && n_items > 0) {
      tc_fence_after();
      float mul;
      if constexpr (C::ROLE == ROLE_FWD) {
        mul = (l_run > 0.f) ? 1.f / l_run : 0.f;
      } else if constexpr (C::ROLE == ROLE_DV) {
        mul = 1.f;
      } else {
        mul = p.scale;
      }
      const int orow = r0 + srow;
      const long long obase = static_cast<long long>(b) * p.out_sb + static_cast<long long>(h) * p.out_sh +
                              static_cast<long long>(orow) * p.out_sn;
#pragma unroll 1
      for (int k = 0; k < C::D / 32; ++k) {
        uint32_t r[32];
        tmem_ld32(tq + 32 * k, r);
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]) * mul;
        if (orow < N) store_out32<C::BF16>(p.out, obase + 32 * k, v, !C::ROWS_ARE_Q && p.out_f32);
      }
      if constexpr (C::ROLE == ROLE_FWD) {
        if (p.lse != nullptr && orow < N) {
          const float LN2 = 0.6931471805599453f;
          p.lse[rowbase_q + orow] = (l_run > 0.f) ? (m_run + __log2f(l_run)) * LN2 : -INFINITY;
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, 512);
  }
}

}  // namespace gqafa
