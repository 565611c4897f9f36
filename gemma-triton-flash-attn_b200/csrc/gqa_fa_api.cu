// Host side of the C ABI declared in include/gqa_fa_b200.h: argument
// validation, TMA tensor-map encoding, per-head_dim kernel configuration and
// launches. Tile shapes are fixed per head_dim (there is no runtime tuning):
//
//   head_dim 256  forward  M=128 BN=128, one 256-column O chunk
//                 dQ, dK   M=128 BN=128, single-buffered scores (TMEM: 256+128+128)
//                 dV       M=128 BN=128, double-buffered scores
//   head_dim 512  all      CTA pairs (attn_pair_kernel.cuh), 64 rows per CTA, BN=256
//   head_dim 64, 128       1-CTA kernels, M=128 BN=128, recomputing backward
#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdarg>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "../../include/gqa_fa_b200.h"
#include "attn_pair_kernel.cuh"
#include "attn_dkv_kernel.cuh"

namespace gqafa {

__device__ int g_status_word;

namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeFn get_encode() {
  static std::once_flag once;
  static EncodeFn fn = nullptr;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeFn>(p);
  });
  return fn;
}

struct TensorDesc {
  const void* ptr;
  long long sb, sh, sn;  // element strides, d stride == 1
  int H;
};

// Validate one [B, H, N, D] tensor and return TMA-legal strides.
int check_tensor(const char* name, const void* ptr, const long long* st, int B, int H, int N, int D,
                 TensorDesc* out) {
  if (ptr == nullptr) return fail(GQAFA_ERR_INVALID, "%s: null pointer", name);
  if (st == nullptr) return fail(GQAFA_ERR_INVALID, "%s: null strides", name);
  if (reinterpret_cast<uintptr_t>(ptr) % 16 != 0)
    return fail(GQAFA_ERR_INVALID, "%s: data pointer must be 16-byte aligned", name);
  if (st[3] != 1) return fail(GQAFA_ERR_INVALID, "%s: last (head_dim) stride must be 1, got %lld", name, st[3]);
  long long sn = st[2], sh = st[1], sb = st[0];
  // Size-1 dims may carry any stride in torch; give TMA a natural one.
  if (N == 1) sn = D;
  if (H == 1) sh = sn * N;
  if (B == 1) sb = sh * H;
  const long long s3[3] = {sn, sh, sb};
  for (int i = 0; i < 3; ++i) {
    if (s3[i] <= 0 || s3[i] % 8 != 0)
      return fail(GQAFA_ERR_INVALID,
                  "%s: strides must be positive multiples of 8 elements (16 bytes), got "
                  "(%lld, %lld, %lld, %lld)",
                  name, st[0], st[1], st[2], st[3]);
    if (s3[i] * 2 >= (1LL << 40)) return fail(GQAFA_ERR_INVALID, "%s: stride too large for TMA", name);
  }
  out->ptr = ptr;
  out->sb = sb;
  out->sh = sh;
  out->sn = sn;
  out->H = H;
  return GQAFA_OK;
}

int encode_map(CUtensorMap* m, const TensorDesc& t, int B, int N, int D, int box_rows, bool bf16) {
  EncodeFn enc = get_encode();
  if (!enc) return fail(GQAFA_ERR_CUDA, "cuTensorMapEncodeTiled unavailable from the driver");
  cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)N, (cuuint64_t)t.H, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)(t.sn * 2), (cuuint64_t)(t.sh * 2), (cuuint64_t)(t.sb * 2)};
  cuuint32_t box[4] = {64u, (cuuint32_t)box_rows, 1u, 1u};
  cuuint32_t estr[4] = {1u, 1u, 1u, 1u};
  CUresult r = enc(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4,
                   const_cast<void*>(t.ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(GQAFA_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return GQAFA_OK;
}

// Make the device of `stream` (or the current device for the legacy stream)
// current on this thread with its primary context bound. Needed because the
// caller may run on a thread where no context is current yet (for example the
// autograd engine's worker thread), and the driver calls below (tensor-map
// encoding) need one.
int bind_device(cudaStream_t stream) {
  int dev = 0;
  cudaError_t e = (stream != nullptr) ? cudaStreamGetDevice(stream, &dev) : cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(GQAFA_ERR_CUDA, "cannot resolve the stream's device: %s", cudaGetErrorString(e));
  e = cudaSetDevice(dev);
  if (e != cudaSuccess) return fail(GQAFA_ERR_CUDA, "cudaSetDevice(%d): %s", dev, cudaGetErrorString(e));
  return GQAFA_OK;
}

// Diagnostics buffer (WC_NUM counters) set by gqafa_set_wait_counters; null = off.
std::atomic<unsigned long long*> g_prof_buffer{nullptr};
// Test knobs set by gqafa_set_test_waits: the launches' wait bound and the
// switch that keeps the TMA producers idle.
std::atomic<long long> g_wait_limit{WAIT_LIMIT_CYCLES};
std::atomic<int> g_no_loads{0};

int* status_ptr() {
  static std::mutex mu;
  static int* ptrs[128] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 128) return nullptr;
  std::lock_guard<std::mutex> lk(mu);
  if (!ptrs[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_status_word) != cudaSuccess) return nullptr;
    ptrs[dev] = static_cast<int*>(p);
  }
  return ptrs[dev];
}

template <class C>
// maps: R1, R2, C1, C2, Y and (pair kernels) the workspace store map; an
// unused slot may hold any valid map.
int launch(const CUtensorMap (&maps)[6], KParams p, cudaStream_t stream) {
  static std::atomic<unsigned long long> attr_done_mask{0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return fail(GQAFA_ERR_CUDA, "cudaGetDevice failed");
  const unsigned long long bit = 1ULL << (dev & 63);
  const void* kfn;
  if constexpr (C::PAIR) {
    kfn = reinterpret_cast<const void*>(&attn_pair_kernel<C>);
  } else {
    kfn = reinterpret_cast<const void*>(&attn_kernel<C>);
  }
  if (!(attr_done_mask.load() & bit)) {
    cudaError_t e = cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
    if (e != cudaSuccess) return fail(GQAFA_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    attr_done_mask.fetch_or(bit);
  }
  // Row range (whole sequence unless a *_rows entry point narrowed it); every
  // kernel's row tile is 128 rows, and range starts are multiples of 128.
  p.tile_begin = p.row_begin / C::MP;
  p.num_row_tiles = (p.row_end + C::MP - 1) / C::MP - p.tile_begin;
  p.prof = g_prof_buffer.load(std::memory_order_relaxed);
  const long long heads = C::ROWS_ARE_Q ? p.Hq : p.Hkv;
  const long long grid = (long long)p.num_row_tiles * heads * p.B * C::NCHUNK * (C::PAIR ? 2 : 1);
  if (grid <= 0 || grid > 0x7fffffffLL) return fail(GQAFA_ERR_INVALID, "grid size %lld out of range", grid);
  if constexpr (C::PAIR) {
    attn_pair_kernel<C><<<(unsigned)grid, C::THREADS, C::SMEM_BYTES, stream>>>(maps[0], maps[1], maps[2], maps[3],
                                                                         maps[4], maps[5], p);
  } else {
    attn_kernel<C><<<(unsigned)grid, 256, C::SMEM_BYTES, stream>>>(maps[0], maps[1], maps[2], maps[3], maps[4], p);
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(GQAFA_ERR_CUDA, "kernel launch: %s", cudaGetErrorString(e));
  return GQAFA_OK;
}

// Fixed configurations. Cfg<ROLE, D, BN, NS, NSTAGES, YGROUP, BF16> (128-row tiles)
template <bool BF16> using Fwd256 = Cfg<ROLE_FWD, 256, 128, 2, 8, 4, BF16>;
template <bool BF16> using Dq256 = Cfg<ROLE_DQ, 256, 128, 1, 6, 2, BF16>;
template <bool BF16> using Dk256 = PairCfg<ROLE_DK, 256, 128, 2, 4, BF16>;  // pair: faster than 1-CTA here
template <bool BF16> using Dv256 = Cfg<ROLE_DV, 256, 128, 2, 8, 4, BF16>;
// head_dim 64 and 128: the 1-CTA template throughout (the whole accumulator
// and double-buffered scores fit one SM's TMEM); the backward recomputes.
template <bool BF16> using Fwd128 = Cfg<ROLE_FWD, 128, 128, 2, 8, 2, BF16>;
template <bool BF16> using Dq128 = Cfg<ROLE_DQ, 128, 128, 1, 8, 2, BF16>;
template <bool BF16> using Dk128 = Cfg<ROLE_DK, 128, 128, 1, 8, 2, BF16>;
template <bool BF16> using Dv128 = Cfg<ROLE_DV, 128, 128, 2, 8, 2, BF16>;
template <bool BF16> using Fwd64 = Cfg<ROLE_FWD, 64, 128, 2, 8, 1, BF16>;
template <bool BF16> using Dq64 = Cfg<ROLE_DQ, 64, 128, 1, 8, 1, BF16>;
template <bool BF16> using Dk64 = Cfg<ROLE_DK, 64, 128, 1, 8, 1, BF16>;
template <bool BF16> using Dv64 = Cfg<ROLE_DV, 64, 128, 2, 8, 1, BF16>;
// head_dim 512: CTA pairs, PairCfg<ROLE, D, BN, NS, NSTAGES, BF16>. The forward keeps all 512 O
// columns in TMEM (256 per CTA), so S is computed once per item. 256-column items make
// every score MMA an N=256 pair instruction (full tensor rate; N=128 pair MMAs run at 70%), at the
// price of single-buffered S/dP in TMEM for dQ and dK (256 + 128 + 128 columns).
template <bool BF16> using Fwd512 = PairCfg<ROLE_FWD, 512, 256, 2, 3, BF16>;
template <bool BF16> using Dq512 = PairCfg<ROLE_DQ, 512, 256, 1, 2, BF16, 2>;
template <bool BF16> using Dk512 = PairCfg<ROLE_DK, 512, 256, 1, 2, BF16>;
template <bool BF16> using Dv512 = PairCfg<ROLE_DV, 512, 256, 2, 3, BF16>;

// Materialised backward (gqafa_bwd_ws): a pair dQ kernel that also stores P
// and dS, then the dK + dV kernel. At head_dim 256 the dQ kernel is the
// pair configuration with 256-key items (the recomputing path keeps the
// 1-CTA Dq256).
template <bool BF16> using Dkv512 = DkvCfg<512, 7, BF16>;
template <bool BF16> using DqWs256 = PairCfg<ROLE_DQ, 256, 256, 1, 4, BF16, 4>;
template <bool BF16> using Dkv256 = DkvCfg<256, 7, BF16>;

struct Problem {
  int B, Hq, Hkv, N, D, causal, window;
  int Nk;  // key length (== N except for the KV-cache forward)
  bool kv_f32;  // dK / dV written as fp32 (gqafa_bwd_partial)
  int row_begin, row_end;  // rows of the row-tile dimension to compute
  float scale;
  bool bf16;
};

int check_problem(int B, int Hq, int Hkv, int N, int D, float scale, int causal, int window, int dtype,
                  Problem* pr) {
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || N <= 0)
    return fail(GQAFA_ERR_INVALID, "sizes must be positive (B=%d H_Q=%d H_KV=%d N=%d)", B, Hq, Hkv, N);
  if (Hq % Hkv != 0) return fail(GQAFA_ERR_INVALID, "H_Q (%d) must be a multiple of H_KV (%d)", Hq, Hkv);
  if (dtype != GQAFA_DTYPE_FP16 && dtype != GQAFA_DTYPE_BF16)
    return fail(GQAFA_ERR_INVALID, "dtype code %d is not fp16 (0) or bf16 (1)", dtype);
  if (D != 64 && D != 128 && D != 256 && D != 512)
    return fail(GQAFA_ERR_UNSUPPORTED, "head_dim %d is not implemented on sm_100a (supported: 64, 128, 256, 512)",
                D);
  if (!(scale > 0.f) || !std::isfinite(scale))
    return fail(GQAFA_ERR_INVALID, "softmax_scale must be positive and finite");
  if (window < 0) return fail(GQAFA_ERR_INVALID, "window must be >= 0");
  pr->B = B;
  pr->Hq = Hq;
  pr->Hkv = Hkv;
  pr->N = N;
  pr->D = D;
  pr->causal = causal ? 1 : 0;
  pr->Nk = N;
  pr->kv_f32 = false;
  // Reference semantics: the window only applies to causal attention and a
  // window covering the whole sequence is plain causal.
  pr->window = (pr->causal && window > 0 && window < N) ? window : 0;
  pr->scale = scale;
  pr->bf16 = (dtype == GQAFA_DTYPE_BF16);
  pr->row_begin = 0;
  pr->row_end = N;
  return GQAFA_OK;
}

KParams base_params(const Problem& pr) {
  KParams p;
  std::memset(&p, 0, sizeof(p));
  p.B = pr.B;
  p.Hq = pr.Hq;
  p.Hkv = pr.Hkv;
  p.N = pr.N;
  p.Nk = pr.Nk;
  p.qoff = pr.Nk - pr.N;
  p.G = pr.Hq / pr.Hkv;
  p.causal = pr.causal;
  p.window = pr.window;
  p.scale = pr.scale;
  p.scale_log2 = pr.scale * 1.4426950408889634f;
  p.row_begin = pr.row_begin;
  p.row_end = pr.row_end;
  p.wait_limit = g_wait_limit.load(std::memory_order_relaxed);
  p.no_loads = g_no_loads.load(std::memory_order_relaxed);
  return p;
}

void set_out(KParams& p, void* ptr, const TensorDesc& t) {
  p.out = ptr;
  p.out_sb = t.sb;
  p.out_sh = t.sh;
  p.out_sn = t.sn;
}

template <bool BF16, class CF>
int fwd_impl(const Problem& pr, const TensorDesc& q, const TensorDesc& k, const TensorDesc& v, void* o,
             const TensorDesc& od, float* lse, cudaStream_t st) {
  CUtensorMap maps[6];
  int rc;
  if ((rc = encode_map(&maps[0], q, pr.B, pr.N, pr.D, CF::M, BF16))) return rc;
  int cbox = CF::BN, ybox = CF::BN;
  if constexpr (CF::PAIR) {
    cbox = CF::C_BOX;
    ybox = CF::Y_BOX;
  }
  if ((rc = encode_map(&maps[2], k, pr.B, pr.Nk, pr.D, cbox, BF16))) return rc;
  if ((rc = encode_map(&maps[4], v, pr.B, pr.Nk, pr.D, ybox, BF16))) return rc;
  maps[1] = maps[0];
  maps[3] = maps[2];
  KParams p = base_params(pr);
  set_out(p, o, od);
  p.lse = lse;
  p.status = status_ptr();
  if (!p.status) return fail(GQAFA_ERR_CUDA, "cannot resolve the device status word");
  maps[5] = maps[0];
  return launch<CF>(maps, p, st);
}

template <bool BF16, class CQ, class CK, class CV>
int bwd_impl(const Problem& pr, const TensorDesc& q, const TensorDesc& k, const TensorDesc& v,
             const TensorDesc& o, const TensorDesc& dout, const float* lse, void* dq, const TensorDesc& dqd,
             void* dk, const TensorDesc& dkd, void* dv, const TensorDesc& dvd, float* delta, cudaStream_t st,
             int stages) {
  int* status = status_ptr();
  if (!status) return fail(GQAFA_ERR_CUDA, "cannot resolve the device status word");
  int rc;
  if (stages & 1) {  // dQ + delta
    CUtensorMap maps[6];
    if ((rc = encode_map(&maps[0], q, pr.B, pr.N, pr.D, CQ::M, BF16))) return rc;
    if ((rc = encode_map(&maps[1], dout, pr.B, pr.N, pr.D, CQ::M, BF16))) return rc;
    if ((rc = encode_map(&maps[2], k, pr.B, pr.N, pr.D, CQ::C_BOX, BF16))) return rc;
    if ((rc = encode_map(&maps[3], v, pr.B, pr.N, pr.D, CQ::C_BOX, BF16))) return rc;
    if ((rc = encode_map(&maps[4], k, pr.B, pr.N, pr.D, CQ::Y_BOX, BF16))) return rc;
    KParams p = base_params(pr);
    set_out(p, dq, dqd);
    p.lse = const_cast<float*>(lse);
    p.delta = delta;
    p.o = o.ptr;
    p.o_sb = o.sb;
    p.o_sh = o.sh;
    p.o_sn = o.sn;
    p.dout = dout.ptr;
    p.do_sb = dout.sb;
    p.do_sh = dout.sh;
    p.do_sn = dout.sn;
    p.status = status;
    if (!p.ws) maps[5] = maps[0];
    if ((rc = launch<CQ>(maps, p, st))) return rc;
  }
  if (stages & 2) {  // dK
    CUtensorMap maps[6];
    if ((rc = encode_map(&maps[0], k, pr.B, pr.N, pr.D, CK::M, BF16))) return rc;
    if ((rc = encode_map(&maps[1], v, pr.B, pr.N, pr.D, CK::M, BF16))) return rc;
    if ((rc = encode_map(&maps[2], q, pr.B, pr.N, pr.D, CK::C_BOX, BF16))) return rc;
    if ((rc = encode_map(&maps[3], dout, pr.B, pr.N, pr.D, CK::C_BOX, BF16))) return rc;
    if ((rc = encode_map(&maps[4], q, pr.B, pr.N, pr.D, CK::Y_BOX, BF16))) return rc;
    KParams p = base_params(pr);
    set_out(p, dk, dkd);
    p.lse = const_cast<float*>(lse);
    p.delta = delta;
    p.status = status;
    p.out_f32 = pr.kv_f32 ? 1 : 0;
    maps[5] = maps[0];
    if ((rc = launch<CK>(maps, p, st))) return rc;
  }
  if (stages & 4) {  // dV
    CUtensorMap maps[6];
    if ((rc = encode_map(&maps[0], k, pr.B, pr.N, pr.D, CV::M, BF16))) return rc;
    if ((rc = encode_map(&maps[2], q, pr.B, pr.N, pr.D, CV::C_BOX, BF16))) return rc;
    if ((rc = encode_map(&maps[4], dout, pr.B, pr.N, pr.D, CV::Y_BOX, BF16))) return rc;
    maps[1] = maps[0];
    maps[3] = maps[2];
    KParams p = base_params(pr);
    set_out(p, dv, dvd);
    p.lse = const_cast<float*>(lse);
    p.delta = delta;
    p.status = status;
    p.out_f32 = pr.kv_f32 ? 1 : 0;
    maps[5] = maps[0];
    if ((rc = launch<CV>(maps, p, st))) return rc;
  }
  return GQAFA_OK;
}

// The materialised backward's workspace as 2 * nblk blocks of [128 queries][256
// keys], 16-bit; boxes of 64 keys x box_rows queries, 128-byte swizzle.
int encode_ws_map(CUtensorMap* m, void* ws, long long nblk, int box_rows, bool bf16) {
  EncodeFn enc = get_encode();
  if (!enc) return fail(GQAFA_ERR_CUDA, "cuTensorMapEncodeTiled unavailable from the driver");
  cuuint64_t dims[3] = {256u, 128u, (cuuint64_t)(2 * nblk)};
  cuuint64_t strides[2] = {256u * 2u, 128u * 256u * 2u};
  cuuint32_t box[3] = {64u, (cuuint32_t)box_rows, 1u};
  cuuint32_t estr[3] = {1u, 1u, 1u};
  CUresult r = enc(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, ws, dims, strides,
                   box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(GQAFA_ERR_CUDA, "cuTensorMapEncodeTiled (workspace) failed (%d)", (int)r);
  return GQAFA_OK;
}

// Blocks of P (and as many of dS) one head stores in the materialised backward.
long long ws_blocks_per_head(const Problem& pr) {
  const int T = (pr.N + 127) / 128;
  int jlo, jn;
  ws_key_blocks(T - 1, pr.N, pr.causal, pr.window, jlo, jn);
  return ws_blocks_before(T - 1, pr.N, pr.causal, pr.window) + jn;
}

long long ws_bytes(const Problem& pr) {
  if (pr.D != 256 && pr.D != 512) return 0;
  return 2LL * pr.B * pr.Hq * ws_blocks_per_head(pr) * (128LL * 256 * 2);
}

// Materialised head_dim-512 backward: stage bit 1 = dQ + delta, writing P and
// dS to the workspace; bit 2 = dK and dV from them.
template <bool BF16, class CQ, class CKV>
int bwd_ws_impl(const Problem& pr, const TensorDesc& q, const TensorDesc& k, const TensorDesc& v,
                const TensorDesc& o, const TensorDesc& dout, const float* lse, void* dq, const TensorDesc& dqd,
                void* dk, const TensorDesc& dkd, void* dv, const TensorDesc& dvd, float* delta, void* ws,
                cudaStream_t st, int stages) {
  int* status = status_ptr();
  if (!status) return fail(GQAFA_ERR_CUDA, "cannot resolve the device status word");
  const long long bph = ws_blocks_per_head(pr);
  const long long nblk = static_cast<long long>(pr.B) * pr.Hq * bph;
  if (2 * nblk > 0x7fffffffLL) return fail(GQAFA_ERR_INVALID, "workspace block count out of range");
  int rc;
  if (stages & 1) {
    CUtensorMap maps[6];
    if ((rc = encode_map(&maps[0], q, pr.B, pr.N, pr.D, CQ::M, BF16))) return rc;
    if ((rc = encode_map(&maps[1], dout, pr.B, pr.N, pr.D, CQ::M, BF16))) return rc;
    if ((rc = encode_map(&maps[2], k, pr.B, pr.N, pr.D, CQ::C_BOX, BF16))) return rc;
    if ((rc = encode_map(&maps[3], v, pr.B, pr.N, pr.D, CQ::C_BOX, BF16))) return rc;
    if ((rc = encode_map(&maps[4], k, pr.B, pr.N, pr.D, CQ::Y_BOX, BF16))) return rc;
    KParams p = base_params(pr);
    set_out(p, dq, dqd);
    p.lse = const_cast<float*>(lse);
    p.delta = delta;
    p.o = o.ptr;
    p.o_sb = o.sb;
    p.o_sh = o.sh;
    p.o_sn = o.sn;
    p.dout = dout.ptr;
    p.do_sb = dout.sb;
    p.do_sh = dout.sh;
    p.do_sn = dout.sn;
    p.ws = ws;
    p.ws_bph = bph;
    p.ws_blocks = nblk;
    p.status = status;
    if ((rc = encode_ws_map(&maps[5], ws, nblk, CQ::M, BF16))) return rc;
    if ((rc = launch<CQ>(maps, p, st))) return rc;
  }
  if (stages & 2) {
    CUtensorMap mws, mq, mdo;
    if ((rc = encode_ws_map(&mws, ws, nblk, 128, BF16))) return rc;
    if ((rc = encode_map(&mq, q, pr.B, pr.N, pr.D, CKV::Y_BOX, BF16))) return rc;
    if ((rc = encode_map(&mdo, dout, pr.B, pr.N, pr.D, CKV::Y_BOX, BF16))) return rc;
    KParams p = base_params(pr);
    set_out(p, dk, dkd);
    p.out2 = dv;
    p.out2_sb = dvd.sb;
    p.out2_sh = dvd.sh;
    p.out2_sn = dvd.sn;
    p.out_f32 = pr.kv_f32 ? 1 : 0;
    p.ws = ws;
    p.ws_bph = bph;
    p.ws_blocks = nblk;
    p.status = status;
    p.tile_begin = 0;
    p.num_row_tiles = (pr.N + CKV::MP - 1) / CKV::MP;
    p.prof = nullptr;
    static std::atomic<unsigned long long> attr_done_mask{0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return fail(GQAFA_ERR_CUDA, "cudaGetDevice failed");
    const unsigned long long bit = 1ULL << (dev & 63);
    if (!(attr_done_mask.load() & bit)) {
      cudaError_t e = cudaFuncSetAttribute(reinterpret_cast<const void*>(&attn_dkv_kernel<CKV>),
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, CKV::SMEM_BYTES);
      if (e != cudaSuccess) return fail(GQAFA_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
      attr_done_mask.fetch_or(bit);
    }
    const long long grid = 2LL * p.num_row_tiles * pr.Hkv * pr.B;
    if (grid > 0x7fffffffLL) return fail(GQAFA_ERR_INVALID, "grid size %lld out of range", grid);
    attn_dkv_kernel<CKV><<<(unsigned)grid, 256, CKV::SMEM_BYTES, st>>>(mws, mq, mdo, p);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(GQAFA_ERR_CUDA, "kernel launch: %s", cudaGetErrorString(e));
  }
  return GQAFA_OK;
}

}  // namespace
}  // namespace gqafa

using namespace gqafa;

// Rows of the row-tile dimension to compute: [row_begin, row_end), row_begin a
// multiple of 128, row_end a multiple of 128 or N.
static int set_rows(Problem* pr, int row_begin, int row_end) {
  if (row_begin < 0 || row_end > pr->N || row_begin >= row_end || row_begin % 128 != 0 ||
      (row_end % 128 != 0 && row_end != pr->N))
    return fail(GQAFA_ERR_INVALID,
                "row range [%d, %d) must satisfy 0 <= begin < end <= N=%d, begin a multiple of 128 and end a "
                "multiple of 128 or N",
                row_begin, row_end, pr->N);
  pr->row_begin = row_begin;
  pr->row_end = row_end;
  return GQAFA_OK;
}

static int fwd_entry(int row_begin, int row_end, const void* q, const long long* q_strides, const void* k,
                     const long long* k_strides, const void* v, const long long* v_strides, void* o,
                     const long long* o_strides, float* lse, int batch, int heads_q, int heads_kv, int seqlen,
                     int head_dim, float softmax_scale, int causal, int window, int dtype, void* stream,
                     int seqlen_k = -1) {
  g_last_error.clear();
  Problem pr{};
  int rc;
  if ((rc = check_problem(batch, heads_q, heads_kv, seqlen, head_dim, softmax_scale, causal, window, dtype, &pr)))
    return rc;
  if (seqlen_k >= 0) {
    if (seqlen_k <= 0) return fail(GQAFA_ERR_INVALID, "key length must be positive");
    if (pr.causal && seqlen_k < seqlen)
      return fail(GQAFA_ERR_INVALID,
                  "causal attention needs key length >= query length (queries are the last %d of %d positions)",
                  seqlen, seqlen_k);
    pr.Nk = seqlen_k;
    pr.window = (pr.causal && window > 0 && window < seqlen_k) ? window : 0;
  }
  if (row_end < 0) row_end = seqlen;
  if ((rc = set_rows(&pr, row_begin, row_end))) return rc;
  TensorDesc qd, kd, vd, od;
  if ((rc = check_tensor("q", q, q_strides, batch, heads_q, seqlen, head_dim, &qd))) return rc;
  if ((rc = check_tensor("k", k, k_strides, batch, heads_kv, pr.Nk, head_dim, &kd))) return rc;
  if ((rc = check_tensor("v", v, v_strides, batch, heads_kv, pr.Nk, head_dim, &vd))) return rc;
  if ((rc = check_tensor("o", o, o_strides, batch, heads_q, seqlen, head_dim, &od))) return rc;
  if (lse != nullptr && reinterpret_cast<uintptr_t>(lse) % 4 != 0)
    return fail(GQAFA_ERR_INVALID, "lse must be 4-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if ((rc = bind_device(st))) return rc;
  if (pr.D == 64)
    return pr.bf16 ? fwd_impl<true, Fwd64<true>>(pr, qd, kd, vd, o, od, lse, st)
                   : fwd_impl<false, Fwd64<false>>(pr, qd, kd, vd, o, od, lse, st);
  if (pr.D == 128)
    return pr.bf16 ? fwd_impl<true, Fwd128<true>>(pr, qd, kd, vd, o, od, lse, st)
                   : fwd_impl<false, Fwd128<false>>(pr, qd, kd, vd, o, od, lse, st);
  if (pr.D == 256)
    return pr.bf16 ? fwd_impl<true, Fwd256<true>>(pr, qd, kd, vd, o, od, lse, st)
                   : fwd_impl<false, Fwd256<false>>(pr, qd, kd, vd, o, od, lse, st);
  return pr.bf16 ? fwd_impl<true, Fwd512<true>>(pr, qd, kd, vd, o, od, lse, st)
                 : fwd_impl<false, Fwd512<false>>(pr, qd, kd, vd, o, od, lse, st);
}

extern "C" int gqafa_fwd(const void* q, const long long* q_strides, const void* k, const long long* k_strides,
                         const void* v, const long long* v_strides, void* o, const long long* o_strides,
                         float* lse, int batch, int heads_q, int heads_kv, int seqlen, int head_dim,
                         float softmax_scale, int causal, int window, int dtype, void* stream) {
  return fwd_entry(0, -1, q, q_strides, k, k_strides, v, v_strides, o, o_strides, lse, batch, heads_q, heads_kv,
                   seqlen, head_dim, softmax_scale, causal, window, dtype, stream);
}

extern "C" int gqafa_fwd_kv(const void* q, const long long* q_strides, const void* k, const long long* k_strides,
                            const void* v, const long long* v_strides, void* o, const long long* o_strides,
                            float* lse, int batch, int heads_q, int heads_kv, int seqlen_q, int seqlen_k,
                            int head_dim, float softmax_scale, int causal, int window, int dtype, void* stream) {
  return fwd_entry(0, -1, q, q_strides, k, k_strides, v, v_strides, o, o_strides, lse, batch, heads_q, heads_kv,
                   seqlen_q, head_dim, softmax_scale, causal, window, dtype, stream, seqlen_k);
}

extern "C" int gqafa_fwd_rows(const void* q, const long long* q_strides, const void* k, const long long* k_strides,
                              const void* v, const long long* v_strides, void* o, const long long* o_strides,
                              float* lse, int batch, int heads_q, int heads_kv, int seqlen, int head_dim,
                              float softmax_scale, int causal, int window, int dtype, void* stream, int row_begin,
                              int row_end) {
  return fwd_entry(row_begin, row_end, q, q_strides, k, k_strides, v, v_strides, o, o_strides, lse, batch, heads_q,
                   heads_kv, seqlen, head_dim, softmax_scale, causal, window, dtype, stream);
}

static int bwd_entry(int stages, int row_begin, int row_end, const void* q, const long long* q_strides, const void* k, const long long* k_strides,
                         const void* v, const long long* v_strides, const void* o, const long long* o_strides,
                         const void* dout, const long long* dout_strides, const float* lse, void* dq,
                         const long long* dq_strides, void* dk, const long long* dk_strides, void* dv,
                         const long long* dv_strides, float* delta, int batch, int heads_q, int heads_kv,
                         int seqlen, int head_dim, float softmax_scale, int causal, int window, int dtype,
                         void* stream, bool kv_f32 = false) {
  g_last_error.clear();
  if (stages <= 0 || stages > 7) return fail(GQAFA_ERR_INVALID, "stage mask %d not in 1..7", stages);
  Problem pr{};
  int rc;
  if ((rc = check_problem(batch, heads_q, heads_kv, seqlen, head_dim, softmax_scale, causal, window, dtype, &pr)))
    return rc;
  pr.kv_f32 = kv_f32;
  if (row_end < 0) row_end = seqlen;
  if ((rc = set_rows(&pr, row_begin, row_end))) return rc;
  TensorDesc qd, kd, vd, od, dod, dqd, dkd, dvd;
  if ((rc = check_tensor("q", q, q_strides, batch, heads_q, seqlen, head_dim, &qd))) return rc;
  if ((rc = check_tensor("k", k, k_strides, batch, heads_kv, seqlen, head_dim, &kd))) return rc;
  if ((rc = check_tensor("v", v, v_strides, batch, heads_kv, seqlen, head_dim, &vd))) return rc;
  if ((rc = check_tensor("o", o, o_strides, batch, heads_q, seqlen, head_dim, &od))) return rc;
  if ((rc = check_tensor("dout", dout, dout_strides, batch, heads_q, seqlen, head_dim, &dod))) return rc;
  if ((rc = check_tensor("dq", dq, dq_strides, batch, heads_q, seqlen, head_dim, &dqd))) return rc;
  if ((rc = check_tensor("dk", dk, dk_strides, batch, heads_kv, seqlen, head_dim, &dkd))) return rc;
  if ((rc = check_tensor("dv", dv, dv_strides, batch, heads_kv, seqlen, head_dim, &dvd))) return rc;
  if (lse == nullptr || delta == nullptr) return fail(GQAFA_ERR_INVALID, "lse and delta must be non-null");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if ((rc = bind_device(st))) return rc;
  if (pr.D == 64)
    return pr.bf16 ? bwd_impl<true, Dq64<true>, Dk64<true>, Dv64<true>>(pr, qd, kd, vd, od, dod, lse, dq, dqd, dk,
                                                                        dkd, dv, dvd, delta, st, stages)
                   : bwd_impl<false, Dq64<false>, Dk64<false>, Dv64<false>>(pr, qd, kd, vd, od, dod, lse, dq, dqd,
                                                                           dk, dkd, dv, dvd, delta, st, stages);
  if (pr.D == 128)
    return pr.bf16 ? bwd_impl<true, Dq128<true>, Dk128<true>, Dv128<true>>(pr, qd, kd, vd, od, dod, lse, dq, dqd,
                                                                           dk, dkd, dv, dvd, delta, st, stages)
                   : bwd_impl<false, Dq128<false>, Dk128<false>, Dv128<false>>(pr, qd, kd, vd, od, dod, lse, dq,
                                                                              dqd, dk, dkd, dv, dvd, delta, st,
                                                                              stages);
  if (pr.D == 256)
    return pr.bf16 ? bwd_impl<true, Dq256<true>, Dk256<true>, Dv256<true>>(pr, qd, kd, vd, od, dod, lse, dq, dqd,
                                                                            dk, dkd, dv, dvd, delta, st, stages)
                   : bwd_impl<false, Dq256<false>, Dk256<false>, Dv256<false>>(pr, qd, kd, vd, od, dod, lse, dq,
                                                                               dqd, dk, dkd, dv, dvd, delta, st, stages);
  return pr.bf16 ? bwd_impl<true, Dq512<true>, Dk512<true>, Dv512<true>>(pr, qd, kd, vd, od, dod, lse, dq, dqd, dk,
                                                                          dkd, dv, dvd, delta, st, stages)
                 : bwd_impl<false, Dq512<false>, Dk512<false>, Dv512<false>>(pr, qd, kd, vd, od, dod, lse, dq, dqd,
                                                                             dk, dkd, dv, dvd, delta, st, stages);
}


#define GQAFA_BWD_PARAMS                                                                                      \
  const void *q, const long long *q_strides, const void *k, const long long *k_strides, const void *v,      \
      const long long *v_strides, const void *o, const long long *o_strides, const void *dout,              \
      const long long *dout_strides, const float *lse, void *dq, const long long *dq_strides, void *dk,     \
      const long long *dk_strides, void *dv, const long long *dv_strides, float *delta, int batch,          \
      int heads_q, int heads_kv, int seqlen, int head_dim, float softmax_scale, int causal, int window,     \
      int dtype, void *stream
#define GQAFA_BWD_ARGS                                                                                        \
  q, q_strides, k, k_strides, v, v_strides, o, o_strides, dout, dout_strides, lse, dq, dq_strides, dk,      \
      dk_strides, dv, dv_strides, delta, batch, heads_q, heads_kv, seqlen, head_dim, softmax_scale, causal, \
      window, dtype, stream

extern "C" int gqafa_bwd(GQAFA_BWD_PARAMS) { return bwd_entry(7, 0, -1, GQAFA_BWD_ARGS); }

extern "C" int gqafa_bwd_stage(int stage, GQAFA_BWD_PARAMS) {
  if (stage < 0 || stage > 2) {
    g_last_error = "stage must be 0 (dQ + delta), 1 (dK) or 2 (dV)";
    return GQAFA_ERR_INVALID;
  }
  return bwd_entry(1 << stage, 0, -1, GQAFA_BWD_ARGS);
}

extern "C" int gqafa_bwd_stage_rows(int stage, GQAFA_BWD_PARAMS, int row_begin, int row_end) {
  if (stage < 0 || stage > 2) {
    g_last_error = "stage must be 0 (dQ + delta), 1 (dK) or 2 (dV)";
    return GQAFA_ERR_INVALID;
  }
  return bwd_entry(1 << stage, row_begin, row_end, GQAFA_BWD_ARGS);
}

extern "C" long long gqafa_bwd_workspace_size(int batch, int heads_q, int heads_kv, int seqlen, int head_dim,
                                              int causal, int window) {
  g_last_error.clear();
  Problem pr{};
  if (check_problem(batch, heads_q, heads_kv, seqlen, head_dim, 1.f, causal, window, GQAFA_DTYPE_BF16, &pr))
    return -1;
  return ws_bytes(pr);
}

static int bwd_ws_entry(int stages, GQAFA_BWD_PARAMS, void* workspace, long long workspace_bytes,
                        bool kv_f32 = false) {
  g_last_error.clear();
  Problem pr{};
  int rc;
  if ((rc = check_problem(batch, heads_q, heads_kv, seqlen, head_dim, softmax_scale, causal, window, dtype, &pr)))
    return rc;
  pr.kv_f32 = kv_f32;
  const long long need = ws_bytes(pr);
  if (need == 0) return bwd_entry(stages == 2 ? 6 : (stages == 1 ? 1 : 7), 0, -1, GQAFA_BWD_ARGS, kv_f32);
  if (workspace == nullptr || workspace_bytes < need)
    return fail(GQAFA_ERR_INVALID, "workspace of %lld bytes needed, got %lld", need, workspace_bytes);
  if (reinterpret_cast<uintptr_t>(workspace) % 256 != 0)
    return fail(GQAFA_ERR_INVALID, "workspace must be 256-byte aligned");
  TensorDesc qd, kd, vd, od, dod, dqd, dkd, dvd;
  if ((rc = check_tensor("q", q, q_strides, batch, heads_q, seqlen, head_dim, &qd))) return rc;
  if ((rc = check_tensor("k", k, k_strides, batch, heads_kv, seqlen, head_dim, &kd))) return rc;
  if ((rc = check_tensor("v", v, v_strides, batch, heads_kv, seqlen, head_dim, &vd))) return rc;
  if ((rc = check_tensor("o", o, o_strides, batch, heads_q, seqlen, head_dim, &od))) return rc;
  if ((rc = check_tensor("dout", dout, dout_strides, batch, heads_q, seqlen, head_dim, &dod))) return rc;
  if ((rc = check_tensor("dq", dq, dq_strides, batch, heads_q, seqlen, head_dim, &dqd))) return rc;
  if ((rc = check_tensor("dk", dk, dk_strides, batch, heads_kv, seqlen, head_dim, &dkd))) return rc;
  if ((rc = check_tensor("dv", dv, dv_strides, batch, heads_kv, seqlen, head_dim, &dvd))) return rc;
  if (lse == nullptr || delta == nullptr) return fail(GQAFA_ERR_INVALID, "lse and delta must be non-null");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if ((rc = bind_device(st))) return rc;
  if (pr.D == 256)
    return pr.bf16 ? bwd_ws_impl<true, DqWs256<true>, Dkv256<true>>(pr, qd, kd, vd, od, dod, lse, dq, dqd, dk, dkd, dv,
                                                                     dvd, delta, workspace, st, stages)
                   : bwd_ws_impl<false, DqWs256<false>, Dkv256<false>>(pr, qd, kd, vd, od, dod, lse, dq, dqd, dk, dkd,
                                                                        dv, dvd, delta, workspace, st, stages);
  return pr.bf16 ? bwd_ws_impl<true, Dq512<true>, Dkv512<true>>(pr, qd, kd, vd, od, dod, lse, dq, dqd, dk, dkd, dv,
                                                                 dvd, delta, workspace, st, stages)
                 : bwd_ws_impl<false, Dq512<false>, Dkv512<false>>(pr, qd, kd, vd, od, dod, lse, dq, dqd, dk, dkd, dv,
                                                                    dvd, delta, workspace, st, stages);
}

extern "C" int gqafa_bwd_ws(GQAFA_BWD_PARAMS, void* workspace, long long workspace_bytes) {
  return bwd_ws_entry(3, GQAFA_BWD_ARGS, workspace, workspace_bytes);
}

extern "C" int gqafa_bwd_partial(GQAFA_BWD_PARAMS, void* workspace, long long workspace_bytes) {
  if (workspace != nullptr && workspace_bytes > 0)
    return bwd_ws_entry(3, GQAFA_BWD_ARGS, workspace, workspace_bytes, true);
  return bwd_entry(7, 0, -1, GQAFA_BWD_ARGS, true);
}

extern "C" int gqafa_bwd_ws_stage(int stage, GQAFA_BWD_PARAMS, void* workspace, long long workspace_bytes) {
  if (stage < 0 || stage > 1) {
    g_last_error = "stage must be 0 (dQ + delta + P/dS) or 1 (dK + dV)";
    return GQAFA_ERR_INVALID;
  }
  return bwd_ws_entry(1 << stage, GQAFA_BWD_ARGS, workspace, workspace_bytes);
}

// ---------------------------------------------------------------------------
// gqafa_bwd_noalloc: the backward for callers that cannot allocate device
// memory. Some callers hold nothing but their input and output tensors: a
// binding that passes only q/k/v/o/dO and the gradient buffers across an FFI,
// or a serving process whose device memory is fully planned up front and
// which may not call cudaMalloc (an allocation can also synchronise the
// device) once it is running. The backward needs one fp32 value per query
// row (delta = rowsum(dO * O)) between its dQ and dK launches, so this entry
// point keeps that workspace in a fixed device array instead of asking the
// caller for it.
//
// The array is a file-scope __device__ variable: every GPU that loads this
// library holds it (4 MiB) until the process exits. Host code cannot use the
// symbol as a pointer, so the first call on each device resolves its device
// address with cudaGetSymbolAddress while that device is current, and caches
// it; make that first call before any CUDA stream capture. All calls share the
// array and it keeps the last call's contents; nothing in it has to start at
// zero, because the dQ launch writes every delta row before the dK launch
// reads it. Two calls whose kernels overlap on the GPU (different streams, no
// ordering between them) race on the array.
// ---------------------------------------------------------------------------
namespace gqafa {
namespace {
constexpr long long kNoAllocDeltaRows = 1LL << 20;  // B * H_Q * N, fp32 each: 4 MiB
static __device__ __align__(256) float g_noalloc_delta[kNoAllocDeltaRows];

float* noalloc_delta_ptr() {
  static std::mutex mu;
  static float* ptrs[128] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 128) {
    fail(GQAFA_ERR_CUDA, "cannot resolve the current device");
    return nullptr;
  }
  std::lock_guard<std::mutex> lk(mu);
  if (!ptrs[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_delta);
    if (e != cudaSuccess) {
      fail(GQAFA_ERR_CUDA, "cudaGetSymbolAddress(no-alloc scratch): %s", cudaGetErrorString(e));
      return nullptr;
    }
    ptrs[dev] = static_cast<float*>(p);
  }
  return ptrs[dev];
}
}  // namespace
}  // namespace gqafa

extern "C" int gqafa_bwd_noalloc(const void* q, const long long* q_strides, const void* k,
                                 const long long* k_strides, const void* v, const long long* v_strides,
                                 const void* o, const long long* o_strides, const void* dout,
                                 const long long* dout_strides, const float* lse, void* dq,
                                 const long long* dq_strides, void* dk, const long long* dk_strides, void* dv,
                                 const long long* dv_strides, int batch, int heads_q, int heads_kv, int seqlen,
                                 int head_dim, float softmax_scale, int causal, int window, int dtype,
                                 void* stream) {
  g_last_error.clear();
  const long long rows = (long long)batch * heads_q * seqlen;
  if (batch > 0 && heads_q > 0 && seqlen > 0 && rows > kNoAllocDeltaRows)
    return fail(GQAFA_ERR_INVALID,
                "gqafa_bwd_noalloc: B*H_Q*N = %lld exceeds the fixed scratch of %lld rows; "
                "use gqafa_bwd with a caller-provided delta buffer",
                rows, kNoAllocDeltaRows);
  int rc;
  if ((rc = bind_device(static_cast<cudaStream_t>(stream)))) return rc;
  float* delta = noalloc_delta_ptr();
  if (!delta) return GQAFA_ERR_CUDA;
  return gqafa_bwd(q, q_strides, k, k_strides, v, v_strides, o, o_strides, dout, dout_strides, lse, dq, dq_strides,
                   dk, dk_strides, dv, dv_strides, delta, batch, heads_q, heads_kv, seqlen, head_dim,
                   softmax_scale, causal, window, dtype, stream);
}

extern "C" int gqafa_supported(int head_dim, int dtype) {
  return (head_dim == 64 || head_dim == 128 || head_dim == 256 || head_dim == 512) &&
         (dtype == GQAFA_DTYPE_FP16 || dtype == GQAFA_DTYPE_BF16);
}

extern "C" int gqafa_set_wait_counters(void* device_counters) {
  g_prof_buffer.store(static_cast<unsigned long long*>(device_counters));
  return GQAFA_OK;
}

extern "C" int gqafa_set_test_waits(long long wait_limit_cycles, int skip_loads) {
  g_wait_limit.store(wait_limit_cycles > 0 ? wait_limit_cycles : WAIT_LIMIT_CYCLES);
  g_no_loads.store(skip_loads ? 1 : 0);
  return GQAFA_OK;
}

extern "C" const char* gqafa_last_error(void) { return g_last_error.c_str(); }

extern "C" int gqafa_device_status(int device, int reset) {
  int prev = 0;
  if (cudaGetDevice(&prev) != cudaSuccess) return -1;
  if (cudaSetDevice(device) != cudaSuccess) return -1;
  int value = -1;
  if (cudaDeviceSynchronize() == cudaSuccess &&
      cudaMemcpyFromSymbol(&value, g_status_word, sizeof(int)) == cudaSuccess) {
    if (reset) {
      const int zero = 0;
      if (cudaMemcpyToSymbol(g_status_word, &zero, sizeof(int)) != cudaSuccess) value = -1;
    }
  } else {
    value = -1;
  }
  cudaSetDevice(prev);
  return value;
}

extern "C" const char* gqafa_version(void) { return "gqa-fa-b200 0.1.0 (sm_100a, tcgen05)"; }
