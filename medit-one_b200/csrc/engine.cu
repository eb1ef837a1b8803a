// MedIT One decode engine for B200 (sm_100a): launch plans, workspace layout, CUDA
// graph capture and the extern "C" boundary declared in include/one_b200.h.
//
// One decode step (the reference's cached forward with s = 1, one/modeling_one.py:
// 671-926) runs, per layer l:
//   row_pre   finish layer l-1 (down_proj partial sums, residual, norm, hx norm),
//             norm_x = norm1(h), running sum S_l += norm_x, mean = S_l / P
//   gemm A    lin1(norm_x) | lin2(hx) | lin3(cx) | cx_moe.gate(clamp(cx))
//   dec_attn  RoPE feature attention, hx_moe / x_moe / cx_moe routers + combine
//             (prompt ingestion: attn_tok, the hx/x gate GEMM, three router launches)
//   gemm C    x_moe -> mean * clamp(.)
//   gemm D    gate_proj / up_proj (row-interleaved) -> gelu(g) * u  |  hx_moe -> hx + clamp(.)
//             |  cx_moe -> cx'
//   gemm E    down_proj, split-K fp32 partials
// then row_pre(final) -> lhs_norm, gemm up_scaler, row_norm (model norm), gemm lm_head
// with a fused argmax. Every launch carries the programmatic-stream-serialization
// attribute; kernels fetch their first weight tiles before griddepcontrol.wait.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/one_b200.h"
#include "common.cuh"
#include "gemm.cuh"
#include "ops.cuh"
#include "rows.cuh"
#include "flash_attn.cuh"
#include "attn_tok.cuh"
#include "router.cuh"
#include "dec_attn.cuh"
#include "sample.cuh"
#include "seq_attn.cuh"

using namespace one;

// ------------------------------------------------------------------ errors
static thread_local std::string g_err;
static int fail(int code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_err = buf;
  return code;
}
#define CK(call)                                                                             \
  do {                                                                                       \
    cudaError_t e_ = (call);                                                                 \
    if (e_ != cudaSuccess) return fail(ONE_ERR_CUDA, "%s: %s (%s:%d)", #call, cudaGetErrorString(e_), __FILE__, __LINE__); \
  } while (0)

extern "C" int one_abi_version(void) { return ONE_B200_ABI_VERSION; }
// error reporting for the library's other translation units (not exported)
extern "C" __attribute__((visibility("hidden"))) int one_set_error(int code, const char* msg) { return fail(code, "%s", msg); }
extern "C" const char* one_last_error(void) { return g_err.c_str(); }

// ------------------------------------------------------------------ TMA descriptors
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// bf16 2-D map over a row-major [rows, cols] array with row stride `ld` elements; box
// {64, box_rows}, 128-byte swizzle, zero fill out of bounds.
static int make_map(CUtensorMap* m, const void* ptr, int rows, int cols, int ld, int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(ONE_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  if ((reinterpret_cast<uintptr_t>(ptr) & 15) || ((size_t)ld * 2) % 16)
    return fail(ONE_ERR_INVALID, "TMA operand must be 16-byte aligned with a 16-byte row stride (ld=%d)", ld);
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  cuuint32_t es[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(ONE_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return ONE_OK;
}

// ------------------------------------------------------------------ GEMM planning
struct ProbSpec {
  int kind = EPI_STORE;
  const void* W = nullptr;
  int Nw = 0, K = 0;
  const void* X = nullptr;
  int ldx = 0;
  const void* bias = nullptr;
  void* out = nullptr;
  int ldo = 0;
  void* out2 = nullptr;
  int ldo2 = 0;
  const void* aux = nullptr;
  int lda = 0;
  float* ws = nullptr;
  int ldw = 0;
  // (first problem's) decode GEMM followed by the attention/router kernel: 64-token tiles with a
  // deep ring on at most one CTA per SM, leaving SMs free for that kernel's prologue
  bool leave_sms = false;
  unsigned long long* best = nullptr;
  int max_splits = 1;
};

enum LaunchKind {
  L_GEMM_TC, L_GEMM_SIMT, L_ROW_PRE, L_ROW_ATTN, L_SCAN, L_ROW_NORM, L_ADVANCE, L_NEXT_IDS,
  L_PROMPT_TAB, L_ATTN_TOK, L_ROUTER, L_ROW_PRE_W, L_DEC_ATTN, L_LM_HEAD, L_SEQ_ATTN
};

struct AdvanceParams {
  int* counters;
  int dpos;
  int dstep;
  int set;
  int pos;
  int step;
};
struct NextIdsParams {
  const unsigned long long* best;
  int* out;
  int T;
};

__global__ void advance_kernel(const AdvanceParams p) {
  pdl_wait();
  if (threadIdx.x == 0) {
    if (p.set) {
      p.counters[0] = p.pos;
      p.counters[1] = p.step;
    } else {
      p.counters[0] += p.dpos;
      p.counters[1] += p.dstep;
    }
  }
}
__global__ void next_ids_kernel(const NextIdsParams p) {
  pdl_wait();
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t < p.T) {
    const unsigned long long key = p.best[t];
    p.out[t] = key ? (int)(0xFFFFFFFFu - (uint32_t)(key & 0xFFFFFFFFull)) : 0;
  }
}

struct Launch {
  LaunchKind kind;
  int bn = 0;       // tensor-core tile width
  int stages = 0;   // ring depth of gemm_bf16_tc_kernel (0: the default for bn)
  int persist = 0;  // gemm_bf16_tc_persistent (one CTA per SM looping over the tiles)
  int minb = 1;  // row_attn: CTAs per SM the instantiation is compiled for
  int grid = 1, block = 1;
  size_t smem = 0;
  int dtype = ONE_DTYPE_BF16;
  int nv = 1;
  GemmParams g;
  SimtGemmParams sg;
  RowPreParams rp;
  RowAttnParams ra;
  ScanParams sc;
  RowNormParams rn;
  AdvanceParams ad;
  NextIdsParams ni;
  PromptTabParams pt;
  DecAttnParams da;
  AttnTokParams at;
  SeqAttnParams sa;
  LmParams lm;
  struct {
    MoeRouter R;
    int n, r, E, k, group;
    unsigned long long tie;
    int np;  // > 0: moe_router_bf16_kernel<np> (input pairs per lane)
    int staged;  // moe_router_bf16_kernel: rows copied ahead by cp.async
  } ro;
};

static int g_num_sms = 0;
static int num_sms() {
  if (!g_num_sms) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
    if (g_num_sms <= 0) g_num_sms = 148;
  }
  return g_num_sms;
}

// Token-tile width: enough CTAs to cover the SMs twice where possible, wider tiles
// (fewer weight re-reads from L2) when the problem already has many weight tiles.
static int pick_bn(int T, int m_tiles_total) {
  if (T >= 8192) return 256;
  if (T >= 2048) return 128;
  for (int bn : {256, 128, 64}) {
    const int ctas = m_tiles_total * ((T + bn - 1) / bn);
    if (bn <= T * 2 && ctas >= num_sms()) return bn;
  }
  // a launch that leaves SMs idle at 64-token tiles: 32-token tiles halve each CTA's epilogue
  // (its MMA chain, K / 16 MMAs, does not depend on the tile width)
  if (m_tiles_total * ((T + 63) / 64) < num_sms()) return 32;
  return T > 32 ? 64 : 32;
}

// Ring depth of the deep per-tile GEMM instantiations (one CTA per SM).
constexpr int kDeepStages = 6;
static int tc_smem(int BN, int stages) {
  if (stages == kDeepStages && BN == 64) return TcCfg<64, kDeepStages>::kSmem;
  switch (BN) {
    case 32: return TcCfg<32>::kSmem;
    case 64: return TcCfg<64>::kSmem;
    case 128: return TcCfg<128>::kSmem;
    default: return TcCfg<256>::kSmem;
  }
}

// Build one GEMM launch over up to four independent problems sharing T tokens.
static int plan_gemm(Launch& L, const ProbSpec* ps, int n, int T, int dtype, DevErr* err) {
  if (n < 1 || n > kMaxProblems) return fail(ONE_ERR_INVALID, "bad problem count");
  memset(&L.g, 0, sizeof(L.g));
  memset(&L.sg, 0, sizeof(L.sg));
  L.dtype = dtype;
  bool tc = dtype == ONE_DTYPE_BF16;
  auto a16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
  for (int i = 0; i < n && tc; ++i) {
    const ProbSpec& s = ps[i];
    // TMA operands: 16-byte aligned rows; vector epilogue: 8-wide rows and chunks
    if (!a16(s.W) || !a16(s.X) || (s.K % 8) || (s.ldx % 8) || (s.Nw % (s.kind == EPI_GELU_UP ? 16 : 8)) ||
        !a16(s.out) || !a16(s.out2) || !a16(s.aux) || !a16(s.bias) || !a16(s.ws) || (s.ldo % 8) || (s.ldo2 % 8) ||
        (s.lda % 8) || (s.ldw % 8))
      tc = false;
  }
  int mt_total = 0;
  for (int i = 0; i < n; ++i) mt_total += (ps[i].Nw + 127) / 128;
  int BN = tc ? pick_bn(T, mt_total) : 64;
  bool deep = false;
  if (tc && ps[0].leave_sms && T <= 256 && mt_total * ((T + 63) / 64) <= num_sms()) {
    int kb = 0;
    for (int i = 0; i < n; ++i) kb = std::max(kb, (ps[i].K + 63) / 64);
    if (kb >= kDeepStages) {
      BN = 64;
      deep = true;
    }
  }
  const int BM = tc ? 128 : 64;
  L.kind = tc ? L_GEMM_TC : L_GEMM_SIMT;
  L.bn = BN;
  int tiles = 0;
  GemmProblem* probs = tc ? L.g.prob : L.sg.prob;
  for (int i = 0; i < n; ++i) {
    const ProbSpec& s = ps[i];
    GemmProblem& P = probs[i];
    P.kind = s.kind;
    P.Nw = s.Nw;
    P.K = s.K;
    P.T = T;
    P.m_tiles = (s.Nw + BM - 1) / BM;
    P.n_tiles = (T + BN - 1) / BN;
    // many token tiles (prompt ingestion): weight tile fastest, so the CTAs running together
    // share activation slabs in L2 (gemm_tile_coords)
    P.m_fast = tc && P.n_tiles >= 2 * num_sms() ? 1 : 0;
    const int kb = (s.K + 63) / 64;
    int splits = 1;
    if (s.kind == EPI_PARTIAL && s.max_splits > 1) {
      const int base = P.m_tiles * P.n_tiles;
      splits = std::min(s.max_splits, std::max(1, (num_sms() + base - 1) / base));
      splits = std::min(splits, std::max(1, kb / 4));
    }
    P.kb_per_split = (kb + splits - 1) / splits;
    P.splits = (kb + P.kb_per_split - 1) / P.kb_per_split;
    P.tile_begin = tiles;
    tiles += P.m_tiles * P.n_tiles * P.splits;
    P.bias = s.bias;
    P.out = s.out;
    P.ldo = s.ldo;
    P.out2 = s.out2;
    P.ldo2 = s.ldo2;
    P.aux = s.aux;
    P.lda = s.lda;
    P.ws = s.ws;
    P.ldw = s.ldw;
    P.best = s.best;
    if (tc) {
      int rc = make_map(&L.g.tmw[i], s.W, s.Nw, s.K, s.K, 128);
      if (rc) return rc;
      rc = make_map(&L.g.tmx[i], s.X, T, s.K, s.ldx, BN);
      if (rc) return rc;
    } else {
      L.sg.w[i] = s.W;
      L.sg.x[i] = s.X;
      L.sg.ldx[i] = s.ldx;
    }
  }
  bool argmax = false;
  for (int i = 0; i < n; ++i) argmax |= ps[i].kind == EPI_ARGMAX;
  if (tc) {
    L.g.nprob = n;
    L.g.total_tiles = tiles;
    L.g.err = err;
    L.block = TcCfg<64>::kThreads;
    if (BN == kPBN && !argmax && tiles >= 2 * num_sms()) {
      L.persist = 1;
      L.smem = PCfg::kSmem;
      L.block = PCfg::kThreads;
      L.grid = num_sms();
      return ONE_OK;
    }
    L.stages = deep ? kDeepStages : 0;
    L.smem = tc_smem(BN, L.stages);
  } else {
    L.sg.nprob = n;
    L.sg.total_tiles = tiles;
    L.block = 256;
    L.smem = 0;
  }
  L.grid = tiles;
  return ONE_OK;
}

// ------------------------------------------------------------------ launching
template <typename... KArgs, typename... Args>
static cudaError_t launch_k(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                            Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  static const bool pdl = [] {
    const char* v = getenv("ONE_B200_NO_PDL");
    return !(v && v[0] == '1');
  }();
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

static bool g_attrs_set = false;
static int set_kernel_attrs() {
  if (g_attrs_set) return ONE_OK;
  CK(cudaFuncSetAttribute(gemm_bf16_tc_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize, TcCfg<32>::kSmem));
  CK(cudaFuncSetAttribute(gemm_bf16_tc_kernel<64, kDeepStages>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                          TcCfg<64, kDeepStages>::kSmem));
  CK(cudaFuncSetAttribute(gemm_bf16_tc_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, TcCfg<64>::kSmem));
  CK(cudaFuncSetAttribute(gemm_bf16_tc_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, TcCfg<128>::kSmem));
  CK(cudaFuncSetAttribute(gemm_bf16_tc_kernel<256>, cudaFuncAttributeMaxDynamicSharedMemorySize, TcCfg<256>::kSmem));
  CK(cudaFuncSetAttribute(gemm_bf16_tc_persistent, cudaFuncAttributeMaxDynamicSharedMemorySize, PCfg::kSmem));
  CK(cudaFuncSetAttribute(lm_head_argmax_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, LmCfg::kSmem));
  CK(cudaFuncSetAttribute(sample_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSampMaxVocab * 4));
  const int attn_max = 220 * 1024;
  CK(cudaFuncSetAttribute(row_attn_kernel<__nv_bfloat16, 16>, cudaFuncAttributeMaxDynamicSharedMemorySize, attn_max));
  CK(cudaFuncSetAttribute(row_attn_kernel<__nv_bfloat16, 16, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                          attn_max));
  CK(cudaFuncSetAttribute(row_attn_kernel<float, 16>, cudaFuncAttributeMaxDynamicSharedMemorySize, attn_max));
  CK(cudaFuncSetAttribute(row_attn_kernel<__nv_bfloat16, 64>, cudaFuncAttributeMaxDynamicSharedMemorySize, attn_max));
  CK(cudaFuncSetAttribute(row_attn_kernel<float, 64>, cudaFuncAttributeMaxDynamicSharedMemorySize, attn_max));
  CK(cudaFuncSetAttribute(moe_router_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, attn_max));
  CK(cudaFuncSetAttribute(moe_router_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, attn_max));
  CK(cudaFuncSetAttribute(flash_attn_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kFaSmem));
  for (int np : {1, 3, 6, 12, 24, 32}) {
    const void* f = np == 1    ? (const void*)moe_router_bf16_kernel<1>
                    : np == 3  ? (const void*)moe_router_bf16_kernel<3>
                    : np == 6  ? (const void*)moe_router_bf16_kernel<6>
                    : np == 12 ? (const void*)moe_router_bf16_kernel<12>
                    : np == 24 ? (const void*)moe_router_bf16_kernel<24>
                               : (const void*)moe_router_bf16_kernel<32>;
    CK(cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
  }
  CK(cudaFuncSetAttribute(dec_attn_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
  CK(cudaFuncSetAttribute(dec_attn_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
  CK(cudaFuncSetAttribute(scan_mean_staged_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kScanSmem));
  CK(cudaFuncSetAttribute(attn_tok_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize, AttnTokSmem<32>::total(16)));
  CK(cudaFuncSetAttribute(attn_tok_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, AttnTokSmem<64>::total(16)));
  g_attrs_set = true;
  return ONE_OK;
}

template <typename T>
static cudaError_t launch_row_pre(const Launch& L, cudaStream_t st) {
  return launch_k(row_pre_kernel<T>, dim3(L.grid), dim3(L.block), 0, st, L.rp);
}
template <typename T>
static cudaError_t launch_row_pre_w(const Launch& L, cudaStream_t st) {
  if (sizeof(T) == 2 && (L.rp.mode == PRE_FIRST || L.rp.splits == 0)) {
    // the first layer, or out0 already holds the MLP residual (unsplit down_proj): packed rows
    switch (L.nv) {
      case 1: return launch_k(row_pre_packed_kernel<1>, dim3(L.grid), dim3(L.block), 0, st, L.rp);
      case 2: return launch_k(row_pre_packed_kernel<2>, dim3(L.grid), dim3(L.block), 0, st, L.rp);
      case 3: return launch_k(row_pre_packed_kernel<3>, dim3(L.grid), dim3(L.block), 0, st, L.rp);
      default: return launch_k(row_pre_packed_kernel<4>, dim3(L.grid), dim3(L.block), 0, st, L.rp);
    }
  }
  switch (L.nv) {
    case 1: return launch_k(row_pre_warp_kernel<T, 1>, dim3(L.grid), dim3(L.block), 0, st, L.rp);
    case 2: return launch_k(row_pre_warp_kernel<T, 2>, dim3(L.grid), dim3(L.block), 0, st, L.rp);
    case 3: return launch_k(row_pre_warp_kernel<T, 3>, dim3(L.grid), dim3(L.block), 0, st, L.rp);
    default: return launch_k(row_pre_warp_kernel<T, 4>, dim3(L.grid), dim3(L.block), 0, st, L.rp);
  }
}
// Prompt ingestion: a warp per token for row_pre when the row fits four 8-element chunks per lane.
static void row_pre_shape(Launch& rp, int D, int T, bool decode) {
  if (!decode && D / 8 <= 128) {
    rp.kind = L_ROW_PRE_W;
    rp.nv = (D / 8 + 31) / 32;
    rp.block = 128;
    rp.grid = (T + 3) / 4;
  } else {
    rp.kind = L_ROW_PRE;
    rp.block = ((D / 8 + 31) / 32) * 32;
    rp.grid = T;
  }
}
template <typename T>
static cudaError_t launch_row_norm(const Launch& L, cudaStream_t st) {
  switch (L.nv) {
    case 1: return launch_k(row_norm_kernel<T, 1>, dim3(L.grid), dim3(L.block), 0, st, L.rn);
    case 2: return launch_k(row_norm_kernel<T, 2>, dim3(L.grid), dim3(L.block), 0, st, L.rn);
    case 3: return launch_k(row_norm_kernel<T, 3>, dim3(L.grid), dim3(L.block), 0, st, L.rn);
    default: return launch_k(row_norm_kernel<T, 4>, dim3(L.grid), dim3(L.block), 0, st, L.rn);
  }
}

static int run(const Launch& L, cudaStream_t st) {
  cudaError_t e = cudaSuccess;
  const bool bf = L.dtype == ONE_DTYPE_BF16;
  switch (L.kind) {
    case L_GEMM_TC:
      if (L.persist) {
        e = launch_k(gemm_bf16_tc_persistent, dim3(L.grid), dim3(L.block), L.smem, st, L.g);
        break;
      }
      switch (L.bn * 100 + L.stages) {
        case 3200: e = launch_k(gemm_bf16_tc_kernel<32>, dim3(L.grid), dim3(L.block), L.smem, st, L.g); break;
        case 6400: e = launch_k(gemm_bf16_tc_kernel<64>, dim3(L.grid), dim3(L.block), L.smem, st, L.g); break;
        case 12800: e = launch_k(gemm_bf16_tc_kernel<128>, dim3(L.grid), dim3(L.block), L.smem, st, L.g); break;
        case 6400 + kDeepStages:
          e = launch_k(gemm_bf16_tc_kernel<64, kDeepStages>, dim3(L.grid), dim3(L.block), L.smem, st, L.g);
          break;
        default: e = launch_k(gemm_bf16_tc_kernel<256>, dim3(L.grid), dim3(L.block), L.smem, st, L.g); break;
      }
      break;
    case L_GEMM_SIMT:
      e = bf ? launch_k(gemm_simt_kernel<__nv_bfloat16>, dim3(L.grid), dim3(L.block), 0, st, L.sg, (DevErr*)nullptr)
             : launch_k(gemm_simt_kernel<float>, dim3(L.grid), dim3(L.block), 0, st, L.sg, (DevErr*)nullptr);
      break;
    case L_ROW_PRE: e = bf ? launch_row_pre<__nv_bfloat16>(L, st) : launch_row_pre<float>(L, st); break;
    case L_ROW_PRE_W: e = bf ? launch_row_pre_w<__nv_bfloat16>(L, st) : launch_row_pre_w<float>(L, st); break;
    case L_ROW_NORM: e = bf ? launch_row_norm<__nv_bfloat16>(L, st) : launch_row_norm<float>(L, st); break;
    case L_ROW_ATTN:
      if (L.nv == 16 && bf && L.minb == 2)
        e = launch_k(row_attn_kernel<__nv_bfloat16, 16, 2>, dim3(L.grid), dim3(L.block), L.smem, st, L.ra);
      else if (L.nv == 16)
        e = bf ? launch_k(row_attn_kernel<__nv_bfloat16, 16>, dim3(L.grid), dim3(L.block), L.smem, st, L.ra)
               : launch_k(row_attn_kernel<float, 16>, dim3(L.grid), dim3(L.block), L.smem, st, L.ra);
      else
        e = bf ? launch_k(row_attn_kernel<__nv_bfloat16, 64>, dim3(L.grid), dim3(L.block), L.smem, st, L.ra)
               : launch_k(row_attn_kernel<float, 64>, dim3(L.grid), dim3(L.block), L.smem, st, L.ra);
      break;
    case L_SCAN:
      if (L.nv == 2) {
        e = launch_k(scan_mean_staged_kernel, dim3(L.grid), dim3(L.block), L.smem, st, L.sc);
        break;
      }
      e = bf ? launch_k(scan_mean_kernel<__nv_bfloat16>, dim3(L.grid), dim3(L.block), 0, st, L.sc)
             : launch_k(scan_mean_kernel<float>, dim3(L.grid), dim3(L.block), 0, st, L.sc);
      break;
    case L_DEC_ATTN:
      e = L.nv == 32 ? launch_k(dec_attn_kernel<32>, dim3(L.grid), dim3(L.block), L.smem, st, L.da)
                     : launch_k(dec_attn_kernel<64>, dim3(L.grid), dim3(L.block), L.smem, st, L.da);
      break;
    case L_PROMPT_TAB: e = launch_k(prompt_table_kernel, dim3(L.grid), dim3(L.block), 0, st, L.pt); break;
    case L_ATTN_TOK:
      switch (L.nv) {
        case 32: e = launch_k(attn_tok_kernel<32>, dim3(L.grid), dim3(L.block), L.smem, st, L.at); break;
        default: e = launch_k(attn_tok_kernel<64>, dim3(L.grid), dim3(L.block), L.smem, st, L.at); break;
      }
      break;
    case L_SEQ_ATTN:
      e = launch_k(seq_attn_kernel, dim3(L.grid, L.sa.H, L.nv), dim3(kSeqThreads), 0, st, L.sa);
      break;
    case L_ROUTER:
      if (L.ro.np > 0) {
        switch (L.ro.np) {
#define ONE_R2(NP)                                                                                                   \
  case NP:                                                                                                           \
    e = launch_k(moe_router_bf16_kernel<NP>, dim3(L.grid), dim3(L.block), L.smem, st, L.ro.R, L.ro.n, L.ro.r, L.ro.E, \
                 L.ro.k, L.ro.group, L.ro.tie, L.ro.staged);                                                         \
    break;
          ONE_R2(1) ONE_R2(3) ONE_R2(6) ONE_R2(12) ONE_R2(24) ONE_R2(32)
#undef ONE_R2
          default: e = cudaErrorInvalidValue; break;
        }
        break;
      }
      e = bf ? launch_k(moe_router_kernel<__nv_bfloat16>, dim3(L.grid), dim3(L.block), L.smem, st, L.ro.R, L.ro.n,
                        L.ro.r, L.ro.E, L.ro.k, L.ro.group, L.ro.tie)
             : launch_k(moe_router_kernel<float>, dim3(L.grid), dim3(L.block), L.smem, st, L.ro.R, L.ro.n, L.ro.r,
                        L.ro.E, L.ro.k, L.ro.group, L.ro.tie);
      break;
    case L_LM_HEAD: e = launch_k(lm_head_argmax_kernel, dim3(L.grid), dim3(L.block), L.smem, st, L.lm); break;
    case L_ADVANCE: e = launch_k(advance_kernel, dim3(1), dim3(32), 0, st, L.ad); break;
    case L_NEXT_IDS: e = launch_k(next_ids_kernel, dim3(L.grid), dim3(L.block), 0, st, L.ni); break;
  }
  if (e != cudaSuccess) return fail(ONE_ERR_CUDA, "kernel launch (kind %d): %s", (int)L.kind, cudaGetErrorString(e));
  return ONE_OK;
}

static int run_plan(const std::vector<Launch>& plan, cudaStream_t st);

// LinearMoE router launch over n tokens with precomputed gate logits (moe_router_kernel).
static int router_np(int in) {
  const int need = (in + 63) / 64;
  for (int np : {1, 3, 6, 12, 24, 32})
    if (need <= np) return np;
  return 0;
}

static int plan_router(Launch& L, const MoeRouter& R, int n, int r, int E, int k, int dtype) {
  auto a4 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 3) == 0; };
  auto a16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
  const int np = router_np(R.in);
  // input rows and gate logits copied 16 bytes at a time: whole 16-byte rows, aligned. Only
  // for wide inputs: the narrow instantiations run three CTAs per SM, which hide the row
  // loads already (staging made the 144-input routers slower, 460 -> 497 us at 262,144 tokens)
  const bool staged = np >= 12 && R.in % 8 == 0 && R.ldx % 8 == 0 && r % 8 == 0 && a16(R.x) && a16(R.glog);
  const Router2Smem L2 = router2_smem(R.in, E, r, staged);
  if (dtype == ONE_DTYPE_BF16 && np > 0 && R.in % 2 == 0 && R.ldx % 2 == 0 && a4(R.x) && a4(R.comb) && a4(R.bias2) &&
      r <= 128 && E <= kMaxExperts && std::min(k, E) <= kR2MaxK && L2.warps >= 1) {
    const void* f = np == 1    ? (const void*)moe_router_bf16_kernel<1>
                    : np == 3  ? (const void*)moe_router_bf16_kernel<3>
                    : np == 6  ? (const void*)moe_router_bf16_kernel<6>
                    : np == 12 ? (const void*)moe_router_bf16_kernel<12>
                    : np == 24 ? (const void*)moe_router_bf16_kernel<24>
                               : (const void*)moe_router_bf16_kernel<32>;
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, f, 32 * L2.warps, L2.total) != cudaSuccess || per_sm < 1)
      return fail(ONE_ERR_CUDA, "router kernel does not fit an SM");
    const int group = std::max(1, std::min(32, n / (num_sms() * per_sm * L2.warps)));
    const int groups = (n + group - 1) / group;
    L.kind = L_ROUTER;
    L.dtype = dtype;
    L.smem = L2.total;
    L.block = 32 * L2.warps;
    L.grid = std::max(1, std::min((groups + L2.warps - 1) / L2.warps, num_sms() * per_sm));
    L.ro.R = R;
    L.ro.n = n;
    L.ro.r = r;
    L.ro.E = E;
    L.ro.k = k;
    L.ro.group = group;
    L.ro.tie = topk_tie_selection(E, std::min(k, E));
    L.ro.np = np;
    L.ro.staged = staged ? 1 : 0;
    return ONE_OK;
  }
  const int es = dtype == ONE_DTYPE_F32 ? 4 : 2;
  const size_t smem = moe_router_smem_bytes(R.in, r, E, es);
  const int warps = moe_router_warps(R.in, r, E, es);
  if (warps < 1 || smem > 220 * 1024) return fail(ONE_ERR_UNSUPPORTED, "router: %zu B of shared memory", smem);
  const int per_sm = std::max(1, std::min(2048 / (32 * warps), (int)((228 * 1024) / (smem + 1024))));
  // tokens per warp group: enough groups for ~24 warps per SM; the selections of a group run
  // one per lane
  const int group = std::max(1, std::min(32, n / (num_sms() * 24)));
  const int groups = (n + group - 1) / group;
  L.kind = L_ROUTER;
  L.dtype = dtype;
  L.smem = smem;
  L.block = 32 * warps;
  L.grid = std::max(1, std::min((groups + warps - 1) / warps, num_sms() * per_sm));
  L.ro.R = R;
  L.ro.n = n;
  L.ro.r = r;
  L.ro.E = E;
  L.ro.k = k;
  L.ro.group = group;
  L.ro.tie = topk_tie_selection(E, std::min(k, E));
  L.ro.np = 0;
  return ONE_OK;
}

// Prompt ingestion takes the warp-per-token attention kernel (attn_tok_kernel) for bf16
// models with an even number of heads <= 16 and head_dim 32 or 64.
// Decode steps of routed bf16 models with the same head shapes take dec_attn_kernel.
static bool dec_attn_eligible(const one_config& c) {
  const int H = c.num_attention_heads, HH = H * H;
  return c.dtype == ONE_DTYPE_BF16 && c.num_experts > 0 && H >= 2 && H <= 16 && H % 2 == 0 &&
         (c.head_dim == 32 || c.head_dim == 64) && c.r % 16 == 0 && c.r <= 128 && HH % 16 == 0 &&
         c.transformer_dim % 8 == 0;
}

static bool attn_tok_eligible(const one_config& c) {
  const int H = c.num_attention_heads, Dh = c.head_dim;
  return c.dtype == ONE_DTYPE_BF16 && H >= 2 && H <= 16 && H % 2 == 0 && (Dh == 32 || Dh == 64);
}

// ------------------------------------------------------------------ workspace layout
struct Layout {
  size_t off = 0;
  size_t take(size_t bytes) {
    size_t o = (off + 1023) & ~size_t(1023);
    off = o + bytes;
    return o;
  }
};

struct Bufs {
  // model dtype [Tm, D] unless noted
  size_t h, norm_x, hx, hx_pre, cx[2], cxc[2], mean, out0, hf, u, hn;
  size_t proj;     // [Tm, 3*HD]
  size_t gcx;      // [Tm, r]
  size_t o;        // [Tm, HH]
  size_t comb_hx, comb_x;  // [Tm, HH]
  size_t comb_cx;  // [Tm, D]
  size_t act;      // [Tm, I]
  size_t ws;       // fp32 [ws_rows, D]
  size_t best;     // u64 [Tm]
  size_t ids_out;  // i32 [Tm]
  size_t hist;     // i32 [hist_cap, Bm]
  size_t state;    // fp32 [L, Bm, D]
  size_t counters; // i32 [4]
  size_t err;      // DevErr
  size_t ridx;     // i32 [Tm, 3, k]
  size_t ghx, gx;  // [Tm, r] hx_moe / x_moe gate logits (prompt ingestion)
  size_t rope;     // bf16 [Tm, head_dim] RoPE cos | sin table of a prompt call
  size_t recip;    // fp32 [Tm][2] a prompt call's prefix-mean divisors and their reciprocals
  size_t total;
  int ws_rows;
};

static constexpr int kMaxSplits = 16;

static Bufs layout(const one_config& c, int max_tokens, int max_batch, int hist_cap) {
  const size_t es = c.dtype == ONE_DTYPE_F32 ? 4 : 2;
  const size_t Tm = (size_t)std::max(max_tokens, max_batch);
  const size_t D = c.transformer_dim, HD = (size_t)c.num_attention_heads * c.head_dim,
               HH = (size_t)c.num_attention_heads * c.num_attention_heads;
  Layout Lo;
  Bufs b;
  b.h = Lo.take(Tm * D * es);
  b.norm_x = Lo.take(Tm * D * es);
  b.hx = Lo.take(Tm * D * es);
  b.hx_pre = Lo.take(Tm * D * es);
  b.cx[0] = Lo.take(Tm * D * es);
  b.cx[1] = Lo.take(Tm * D * es);
  b.cxc[0] = Lo.take(Tm * D * es);
  b.cxc[1] = Lo.take(Tm * D * es);
  b.mean = Lo.take(Tm * D * es);
  b.out0 = Lo.take(Tm * D * es);
  b.hf = Lo.take(Tm * D * es);
  b.u = Lo.take(Tm * (size_t)c.hidden_size * es);
  b.hn = Lo.take(Tm * (size_t)c.hidden_size * es);
  b.proj = Lo.take(Tm * 3 * HD * es);
  b.gcx = Lo.take(Tm * (size_t)std::max(c.r, 1) * es);
  b.o = Lo.take(Tm * HH * es);
  b.comb_hx = Lo.take(Tm * HH * es);
  b.comb_x = Lo.take(Tm * HH * es);
  b.comb_cx = Lo.take(Tm * D * es);
  b.act = Lo.take(Tm * (size_t)c.intermediate_size * es);
  b.ws_rows = std::max(kMaxSplits * max_batch, max_tokens);
  b.ws = Lo.take((size_t)b.ws_rows * D * 4);
  b.best = Lo.take(Tm * 8);
  b.ids_out = Lo.take(Tm * 4);
  b.hist = Lo.take((size_t)std::max(hist_cap, 1) * max_batch * 4);
  b.state = Lo.take((size_t)c.num_hidden_layers * max_batch * D * 4);
  b.counters = Lo.take(16);
  b.err = Lo.take(sizeof(DevErr));
  b.ridx = Lo.take(Tm * 3 * (size_t)std::max(c.top_k, 1) * 4);
  b.ghx = Lo.take(Tm * (size_t)std::max(c.r, 1) * es);
  b.gx = Lo.take(Tm * (size_t)std::max(c.r, 1) * es);
  b.rope = Lo.take(Tm * (size_t)c.head_dim * 2);
  b.recip = Lo.take(Tm * 8);
  b.total = Lo.take(0) + 1024;
  return b;
}

// ------------------------------------------------------------------ engine
struct one_engine {
  one_config c;
  std::vector<const void*> gw;
  std::vector<const void*> lw;
  uint8_t* ws = nullptr;
  Bufs b;
  int max_tokens = 0, max_batch = 0, hist_cap = 0;
  const float* inv_freq = nullptr;
  const float* ddiv = nullptr;
  int div_len = 0;
  // graphs: the multi-step greedy graph (one_engine_capture) and one-step graphs per
  // (batch, ids, logits, next_ids) used by one_engine_step. Captured on an engine-owned
  // stream (the legacy default stream cannot be captured), launched on the caller's.
  cudaStream_t cap_stream = nullptr;
  cudaGraphExec_t graph = nullptr;
  cudaGraph_t graph_def = nullptr;
  struct StepGraph {
    int batch;
    const int* ids;
    void* logits;
    int* next_ids;
    cudaGraph_t g;
    cudaGraphExec_t x;
  };
  std::vector<StepGraph> step_graphs;
  bool use_graphs = true;
  template <typename P = void>
  P* at(size_t off) { return reinterpret_cast<P*>(ws + off); }
  const void* L(int l, int slot) const { return lw[(size_t)l * ONE_W_LAYER_SLOTS + slot]; }
};

static int es_of(const one_config& c) { return c.dtype == ONE_DTYPE_F32 ? 4 : 2; }

extern "C" size_t one_engine_workspace_bytes(const one_config* cfg, int32_t max_tokens, int32_t max_batch, int32_t hist_cap) {
  if (!cfg) return 0;
  return layout(*cfg, max_tokens, max_batch, hist_cap).total;
}

static int check_cfg(const one_config& c) {
  if (c.dtype != ONE_DTYPE_BF16 && c.dtype != ONE_DTYPE_F32) return fail(ONE_ERR_INVALID, "dtype must be bf16 or fp32");
  if (c.transformer_dim != c.hidden_size)
    return fail(ONE_ERR_UNSUPPORTED, "transformer_dim (%d) != hidden_size (%d): the pooled path is not built",
                c.transformer_dim, c.hidden_size);
  if (c.transformer_dim % 8 || c.transformer_dim > 1024)
    return fail(ONE_ERR_UNSUPPORTED, "transformer_dim must be a multiple of 8 and <= 1024");
  if (c.num_attention_heads * c.head_dim != c.transformer_dim)
    return fail(ONE_ERR_UNSUPPORTED, "num_attention_heads * head_dim must equal transformer_dim");
  if (c.head_dim % 16 || c.head_dim > 256) return fail(ONE_ERR_UNSUPPORTED, "head_dim must be a multiple of 16, <= 256");
  if (c.num_attention_heads > 64) return fail(ONE_ERR_UNSUPPORTED, "at most 64 heads");
  if (c.num_experts < 0 || c.num_experts > kMaxExperts) return fail(ONE_ERR_UNSUPPORTED, "at most %d experts", kMaxExperts);
  if (c.num_experts > 0 && (c.top_k < 1 || c.r < 1)) return fail(ONE_ERR_INVALID, "top_k and r must be positive");
  if (c.intermediate_size % 8) return fail(ONE_ERR_UNSUPPORTED, "intermediate_size must be a multiple of 8");
  if (c.use_flash_attention && !(dec_attn_eligible(c) && attn_tok_eligible(c) && c.num_attention_heads <= kSeqMaxH))
    return fail(ONE_ERR_UNSUPPORTED,
                "use_flash_attention is built for bf16 models with routed LinearMoE layers, an even number of heads "
                "<= %d and head_dim 32 or 64", kSeqMaxH);
  return ONE_OK;
}

extern "C" int one_engine_create(const one_config* cfg, const void* const* global_w, const void* const* layer_w,
                                 void* workspace, size_t workspace_bytes, int32_t max_tokens, int32_t max_batch,
                                 int32_t hist_cap, const float* inv_freq, const float* decode_div, int32_t div_len,
                                 one_engine** out) {
  if (!cfg || !global_w || !layer_w || !workspace || !out || !inv_freq || !decode_div)
    return fail(ONE_ERR_INVALID, "null argument");
  int rc = check_cfg(*cfg);
  if (rc) return rc;
  if (max_tokens < 1 || max_batch < 1 || div_len < 1) return fail(ONE_ERR_INVALID, "sizes must be positive");
  Bufs b = layout(*cfg, max_tokens, max_batch, hist_cap);
  if (workspace_bytes < b.total) return fail(ONE_ERR_INVALID, "workspace too small: %zu < %zu", workspace_bytes, b.total);
  if (reinterpret_cast<uintptr_t>(workspace) & 1023) return fail(ONE_ERR_INVALID, "workspace must be 1024-byte aligned");
  rc = set_kernel_attrs();
  if (rc) return rc;
  one_engine* e = new one_engine();
  e->c = *cfg;
  e->gw.assign(global_w, global_w + ONE_G_SLOTS);
  e->lw.assign(layer_w, layer_w + (size_t)cfg->num_hidden_layers * ONE_W_LAYER_SLOTS);
  e->ws = reinterpret_cast<uint8_t*>(workspace);
  e->b = b;
  e->max_tokens = max_tokens;
  e->max_batch = max_batch;
  e->hist_cap = hist_cap;
  e->inv_freq = inv_freq;
  e->ddiv = decode_div;
  e->div_len = div_len;
  const char* ng = getenv("ONE_B200_NO_GRAPH");
  e->use_graphs = !(ng && ng[0] == '1');
  cudaError_t ce = cudaStreamCreateWithFlags(&e->cap_stream, cudaStreamNonBlocking);
  if (ce == cudaSuccess) ce = cudaMemset(e->ws + b.counters, 0, 16);
  if (ce == cudaSuccess) ce = cudaMemset(e->ws + b.err, 0, sizeof(DevErr));
  if (ce == cudaSuccess) ce = cudaMemset(e->ws + b.best, 0, (size_t)std::max(max_tokens, max_batch) * 8);
  if (ce != cudaSuccess) {
    delete e;
    return fail(ONE_ERR_CUDA, "workspace init: %s", cudaGetErrorString(ce));
  }
  *out = e;
  return ONE_OK;
}

extern "C" int one_engine_destroy(one_engine* e) {
  if (!e) return ONE_OK;
  if (e->graph) cudaGraphExecDestroy(e->graph);
  if (e->graph_def) cudaGraphDestroy(e->graph_def);
  for (auto& sg : e->step_graphs) {
    cudaGraphExecDestroy(sg.x);
    cudaGraphDestroy(sg.g);
  }
  if (e->cap_stream) cudaStreamDestroy(e->cap_stream);
  delete e;
  return ONE_OK;
}

// Capture `reps` back-to-back runs of `plan` into an executable graph.
static int capture_plan(one_engine* e, const std::vector<Launch>& plan, int reps, cudaGraph_t* g_out,
                        cudaGraphExec_t* x_out) {
  cudaStream_t st = e->cap_stream;
  CK(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
  int rc = ONE_OK;
  for (int s = 0; s < reps && rc == ONE_OK; ++s) rc = run_plan(plan, st);
  cudaGraph_t g = nullptr;
  cudaError_t ce = cudaStreamEndCapture(st, &g);
  if (rc) {
    if (g) cudaGraphDestroy(g);
    return rc;
  }
  if (ce != cudaSuccess) return fail(ONE_ERR_CUDA, "capture: %s", cudaGetErrorString(ce));
  cudaGraphExec_t x = nullptr;
  ce = cudaGraphInstantiate(&x, g, 0);
  if (ce != cudaSuccess) {
    cudaGraphDestroy(g);
    return fail(ONE_ERR_CUDA, "graph instantiate: %s", cudaGetErrorString(ce));
  }
  *g_out = g;
  *x_out = x;
  return ONE_OK;
}

extern "C" int one_engine_reset(one_engine* e, int32_t batch, int32_t pos, void* stream) {
  if (!e || batch < 1 || batch > e->max_batch) return fail(ONE_ERR_INVALID, "bad batch");
  cudaStream_t st = (cudaStream_t)stream;
  const size_t D = e->c.transformer_dim;
  for (int l = 0; l < e->c.num_hidden_layers; ++l)
    CK(cudaMemsetAsync(e->at<float>(e->b.state) + (size_t)l * e->max_batch * D, 0, (size_t)batch * D * 4, st));
  CK(cudaMemsetAsync(e->ws + e->b.best, 0, (size_t)std::max(e->max_tokens, e->max_batch) * 8, st));
  Launch a;
  a.kind = L_ADVANCE;
  a.ad = AdvanceParams{e->at<int>(e->b.counters), 0, 0, 1, pos, 0};
  return run(a, st);
}

// Layer-l weight helper
#define LW(slot) e->L(l, slot)

// Append the kernels of the layer stack for T tokens (decode: T = batch, one token per
// sequence; prefill: T = batch * seq_len).
static int build_layers(one_engine* e, std::vector<Launch>& plan, int T, bool decode, int seq_len, int batch,
                        const int* ids, bool ids_from_best, const float* prompt_div) {
  const one_config& c = e->c;
  const int D = c.transformer_dim, H = c.num_attention_heads, Dh = c.head_dim, HD = H * Dh, HH = H * H;
  const int I = c.intermediate_size;
  const bool moe = c.num_experts > 0;
  const int dt = c.dtype;
  const int nv = (D / 8 + 31) / 32;
  DevErr* err = e->at<DevErr>(e->b.err);
  auto B_ = [&](size_t off) { return e->at<void>(off); };
  const int* counters = e->at<int>(e->b.counters);
  const int es = es_of(c);
  const bool tok = !decode && attn_tok_eligible(c);
  // bf16 prompt ingestion: per-position tables shared by every layer (prefix-mean divisor
  // reciprocals; the RoPE cos / sin for the warp-per-token attention)
  const bool recip = !decode && dt == ONE_DTYPE_BF16;
  if (recip) {
    Launch pt;
    pt.kind = L_PROMPT_TAB;
    pt.block = 256;
    const int half = tok ? Dh / 2 : 0;
    pt.grid = (seq_len * std::max(half, 1) + 255) / 256;
    pt.pt = PromptTabParams{counters, e->inv_freq, seq_len, half, e->at<__nv_bfloat16>(e->b.rope), prompt_div,
                            e->at<float2>(e->b.recip)};
    plan.push_back(pt);
  }
  for (int l = 0; l < c.num_hidden_layers; ++l) {
    const int cur = l & 1, nxt = cur ^ 1;
    // ---- row_pre
    Launch rp;
    rp.dtype = dt;
    rp.nv = nv;
    row_pre_shape(rp, D, T, decode);
    RowPreParams& p = rp.rp;
    memset(&p, 0, sizeof(p));
    p.T = T;
    p.D = D;
    p.vocab = c.vocab_size;
    p.mode = l == 0 ? PRE_FIRST : PRE_MID;
    p.ids_from_best = ids_from_best ? 1 : 0;
    p.decode = decode ? 1 : 0;
    p.ids = ids;
    p.best = e->at<unsigned long long>(e->b.best);
    p.ids_out = e->at<int>(e->b.ids_out);
    p.hist = decode ? e->at<int>(e->b.hist) : nullptr;
    p.hist_cap = e->hist_cap;
    p.counters = counters;
    p.emb = e->gw[ONE_G_EMBED];
    p.div = e->ddiv;
    p.div_len = e->div_len;
    p.ws = e->at<float>(e->b.ws);
    p.out0 = B_(e->b.out0);
    p.hx_pre = B_(e->b.hx_pre);
    if (l > 0) {
      p.prev_norm_w = e->L(l - 1, ONE_W_NORM_W);
      p.prev_norm_b = e->L(l - 1, ONE_W_NORM_B);
    }
    p.norm1_w = LW(ONE_W_NORM1);
    p.h = B_(e->b.h);
    p.norm_x = B_(e->b.norm_x);
    p.hx = B_(e->b.hx);
    p.cx = B_(e->b.cx[cur]);
    p.cxc = B_(e->b.cxc[cur]);
    p.S = e->at<float>(e->b.state) + (size_t)l * e->max_batch * D;
    p.mean = B_(e->b.mean);
    p.err = err;
    if (l > 0 && c.mlp_bias) p.down_b = e->L(l - 1, ONE_W_DOWN_B);
    plan.push_back(rp);  // `splits` of the previous down_proj is filled in by link_splits
    // ---- prefill prefix mean
    if (!decode) {
      Launch s;
      s.kind = L_SCAN;
      s.dtype = dt;
      s.block = 128;
      s.grid = (batch * (D / 2) + 127) / 128;  // one thread per (sequence, feature pair)
      s.sc = ScanParams{batch, seq_len, D, B_(e->b.norm_x), B_(e->b.mean),
                        e->at<float>(e->b.state) + (size_t)l * e->max_batch * D, prompt_div,
                        recip ? e->at<float2>(e->b.recip) : nullptr};
      if (recip && dt == ONE_DTYPE_BF16 && D % kScanFeat == 0) {
        // staged through shared memory: a CTA per (sequence, 128 features)  (nv = 2)
        s.nv = 2;
        s.block = kScanThreads;
        s.grid = batch * (D / kScanFeat);
        s.smem = kScanSmem;
      }
      plan.push_back(s);
    }
    // ---- gemm A
    {
      ProbSpec ps[4];
      int n = 0;
      ps[n].W = LW(ONE_W_LIN1_W); ps[n].Nw = HD; ps[n].K = D; ps[n].X = B_(e->b.norm_x); ps[n].ldx = D;
      ps[n].bias = LW(ONE_W_LIN1_B); ps[n].out = B_(e->b.proj); ps[n].ldo = 3 * HD; ++n;
      ps[n].W = LW(ONE_W_LIN2_W); ps[n].Nw = HD; ps[n].K = D; ps[n].X = B_(e->b.hx); ps[n].ldx = D;
      ps[n].bias = LW(ONE_W_LIN2_B); ps[n].out = e->at<uint8_t>(e->b.proj) + (size_t)HD * es; ps[n].ldo = 3 * HD; ++n;
      ps[n].W = LW(ONE_W_LIN3_W); ps[n].Nw = HD; ps[n].K = D; ps[n].X = B_(e->b.cx[cur]); ps[n].ldx = D;
      ps[n].bias = LW(ONE_W_LIN3_B); ps[n].out = e->at<uint8_t>(e->b.proj) + (size_t)2 * HD * es; ps[n].ldo = 3 * HD; ++n;
      if (moe) {
        ps[n].W = LW(ONE_W_CX_GATE); ps[n].Nw = c.r; ps[n].K = D; ps[n].X = B_(e->b.cxc[cur]); ps[n].ldx = D;
        ps[n].bias = nullptr; ps[n].out = B_(e->b.gcx); ps[n].ldo = c.r; ++n;
      }
      ps[0].leave_sms = decode && dec_attn_eligible(c);
      Launch g;
      int rc = plan_gemm(g, ps, n, T, dt, err);
      if (rc) return rc;
      plan.push_back(g);
    }
    // ---- attention + routers, prompt ingestion: warp-per-token attention writes o (the
    // LinearMoE-clamped copy when routed), then the hx_moe / x_moe gate logits on the tensor
    // cores and one router launch per LinearMoE
    if (decode && dec_attn_eligible(c)) {
      Launch a;
      a.kind = L_DEC_ATTN;
      a.dtype = dt;
      a.nv = Dh;
      a.block = kDecThreads;
      a.smem = Dh == 32 ? dec_layout<32>(H, c.r, c.num_experts, D).total : dec_layout<64>(H, c.r, c.num_experts, D).total;
      if (a.smem > 200 * 1024) return fail(ONE_ERR_UNSUPPORTED, "decode attention/router tile exceeds shared memory");
      a.grid = std::max(1, std::min((T + 1) / 2, num_sms()));
      DecAttnParams& q = a.da;
      memset(&q, 0, sizeof(q));
      q.T = T; q.H = H; q.r = c.r; q.E = c.num_experts; q.k = c.top_k;
      q.counters = counters;
      q.inv_freq = e->inv_freq;
      q.proj = e->at<__nv_bfloat16>(e->b.proj);
      q.scale = 1.0f / sqrtf((float)Dh);
      const __nv_bfloat16 sb = __float2bfloat16_rn(q.scale);
      q.scale_exact = __bfloat162float(sb) == q.scale ? 1 : 0;
      uint16_t sbits;
      memcpy(&sbits, &sb, 2);
      q.scale2 = (uint32_t)sbits * 0x10001u;
      q.wq = (const __nv_bfloat16*)LW(ONE_W_LINQ_W); q.bq = (const __nv_bfloat16*)LW(ONE_W_LINQ_B);
      q.wk = (const __nv_bfloat16*)LW(ONE_W_LINK_W); q.bk = (const __nv_bfloat16*)LW(ONE_W_LINK_B);
      q.wv = (const __nv_bfloat16*)LW(ONE_W_LINV_W); q.bv = (const __nv_bfloat16*)LW(ONE_W_LINV_B);
      const int k = c.top_k;
      int* ridx = e->at<int>(e->b.ridx);
      MoeRouter& r0 = q.rt[0];
      r0.gate_w = LW(ONE_W_HX_GATE); r0.experts = LW(ONE_W_HX_EXPERTS); r0.bias2 = LW(ONE_W_HX_BIAS2);
      r0.in = HH; r0.comb = B_(e->b.comb_hx); r0.idx_out = ridx;
      MoeRouter& r1 = q.rt[1];
      r1.gate_w = LW(ONE_W_X_GATE); r1.experts = LW(ONE_W_X_EXPERTS); r1.bias2 = LW(ONE_W_X_BIAS2);
      r1.in = HH; r1.comb = B_(e->b.comb_x); r1.idx_out = ridx + (size_t)T * k;
      MoeRouter& r2 = q.rt[2];
      r2.glog = B_(e->b.gcx); r2.experts = LW(ONE_W_CX_EXPERTS); r2.bias2 = LW(ONE_W_CX_BIAS2);
      r2.x = B_(e->b.cxc[cur]); r2.ldx = D; r2.in = D; r2.comb = B_(e->b.comb_cx);
      r2.idx_out = ridx + (size_t)2 * T * k;
      q.tie = topk_tie_selection(c.num_experts, std::min(c.top_k, c.num_experts));
      q.err = err;
      // use_flash_attention: the causal attention of a one-token call sees that token only
      q.mode = c.use_flash_attention ? kAttnValue : kAttnFeature;
      plan.push_back(a);
    } else if (tok) {
      Launch a;
      a.kind = L_ATTN_TOK;
      a.dtype = dt;
      a.nv = Dh;
      a.block = kTokWarps * 32;
      AttnTokParams& q = a.at;
      memset(&q, 0, sizeof(q));
      q.T = T; q.H = H; q.seq_len = seq_len;
      q.rope = e->at<__nv_bfloat16>(e->b.rope);
      q.proj = e->at<__nv_bfloat16>(e->b.proj);
      q.scale = 1.0f / sqrtf((float)Dh);
      const __nv_bfloat16 sb = __float2bfloat16_rn(q.scale);
      q.scale_exact = __bfloat162float(sb) == q.scale ? 1 : 0;
      uint16_t sbits;
      memcpy(&sbits, &sb, 2);
      q.scale2 = (uint32_t)sbits * 0x10001u;
      q.wq = (const __nv_bfloat16*)LW(ONE_W_LINQ_W); q.bq = (const __nv_bfloat16*)LW(ONE_W_LINQ_B);
      q.wk = (const __nv_bfloat16*)LW(ONE_W_LINK_W); q.bk = (const __nv_bfloat16*)LW(ONE_W_LINK_B);
      q.wv = (const __nv_bfloat16*)LW(ONE_W_LINV_W); q.bv = (const __nv_bfloat16*)LW(ONE_W_LINV_B);
      q.out = e->at<__nv_bfloat16>(e->b.o);
      // bf16(1e4) = 9984: the clamp bound of a bf16 tensor
      q.clamp2 = moe ? 0x461c461cu : 0u;
      q.mode = kAttnFeature;
      q.out_ld = HH;
      if (c.use_flash_attention) {
        // q | k | v of each token written over its own (already consumed) projection row,
        // then the causal attention across each prompt's tokens writes o
        q.mode = kAttnQKV;
        q.out = e->at<__nv_bfloat16>(e->b.proj);
        q.out_ld = 3 * HD;
      }
      a.smem = Dh == 32 ? AttnTokSmem<32>::total(H) : AttnTokSmem<64>::total(H);
      int per_sm = 1;
      cudaError_t oe = Dh == 32 ? cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, attn_tok_kernel<32>, a.block, a.smem)
                                : cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, attn_tok_kernel<64>, a.block, a.smem);
      if (oe != cudaSuccess || per_sm < 1) return fail(ONE_ERR_CUDA, "attention kernel does not fit an SM");
      a.grid = std::max(1, std::min((T + kTokWarps - 1) / kTokWarps, num_sms() * per_sm));
      plan.push_back(a);
      if (c.use_flash_attention) {
        if (H > kSeqMaxH || seq_len < 1 || T != batch * seq_len)
          return fail(ONE_ERR_UNSUPPORTED, "flash attention: at most %d heads", kSeqMaxH);
        Launch sq;
        sq.kind = L_SEQ_ATTN;
        sq.dtype = dt;
        sq.grid = (seq_len + kSeqQ - 1) / kSeqQ;
        sq.nv = batch;
        sq.block = kSeqThreads;
        sq.sa = SeqAttnParams{e->at<__nv_bfloat16>(e->b.proj), 3 * HD, e->at<__nv_bfloat16>(e->b.o), seq_len, H,
                              1.0f / sqrtf((float)H), moe ? 9984.0f : 0.0f};
        plan.push_back(sq);
      }
      if (moe) {
        ProbSpec ps[2];
        ps[0].W = LW(ONE_W_HX_GATE); ps[0].Nw = c.r; ps[0].K = HH; ps[0].X = B_(e->b.o); ps[0].ldx = HH;
        ps[0].bias = nullptr; ps[0].out = B_(e->b.ghx); ps[0].ldo = c.r;
        ps[1].W = LW(ONE_W_X_GATE); ps[1].Nw = c.r; ps[1].K = HH; ps[1].X = B_(e->b.o); ps[1].ldx = HH;
        ps[1].bias = nullptr; ps[1].out = B_(e->b.gx); ps[1].ldo = c.r;
        Launch g;
        int rc = plan_gemm(g, ps, 2, T, dt, err);
        if (rc) return rc;
        plan.push_back(g);
        const int k = c.top_k;
        int* ridx = e->at<int>(e->b.ridx);
        MoeRouter R[3];
        memset(R, 0, sizeof(R));
        R[0].glog = B_(e->b.ghx); R[0].experts = LW(ONE_W_HX_EXPERTS); R[0].bias2 = LW(ONE_W_HX_BIAS2);
        R[0].x = B_(e->b.o); R[0].ldx = HH; R[0].in = HH; R[0].comb = B_(e->b.comb_hx); R[0].idx_out = ridx;
        R[1].glog = B_(e->b.gx); R[1].experts = LW(ONE_W_X_EXPERTS); R[1].bias2 = LW(ONE_W_X_BIAS2);
        R[1].x = B_(e->b.o); R[1].ldx = HH; R[1].in = HH; R[1].comb = B_(e->b.comb_x);
        R[1].idx_out = ridx + (size_t)T * k;
        R[2].glog = B_(e->b.gcx); R[2].experts = LW(ONE_W_CX_EXPERTS); R[2].bias2 = LW(ONE_W_CX_BIAS2);
        R[2].x = B_(e->b.cxc[cur]); R[2].ldx = D; R[2].in = D; R[2].comb = B_(e->b.comb_cx);
        R[2].idx_out = ridx + (size_t)2 * T * k;
        for (int i = 0; i < 3; ++i) {
          Launch rl;
          rc = plan_router(rl, R[i], T, c.r, c.num_experts, k, dt);
          if (rc) return rc;
          plan.push_back(rl);
        }
      }
    } else {
      if (c.use_flash_attention)
        return fail(ONE_ERR_UNSUPPORTED, "use_flash_attention needs the bf16 warp-per-token / decode attention kernels");
      Launch a;
            a.kind = L_ROW_ATTN;
      a.dtype = dt;
      a.block = kAttnThreads;
      a.grid = std::min((T + kAttnTok - 1) / kAttnTok, num_sms() * 2);
      a.nv = H <= 16 ? 16 : 64;
      a.smem = attn_layout(H, Dh, c.r, c.num_experts, D, moe ? 1 : 0, es, 1).total;
      // prompt ingestion (more token pairs than one CTA per SM covers): two CTAs per SM,
      // without the staged projection / gate weights
      const size_t smem2 = attn_layout(H, Dh, c.r, c.num_experts, D, moe ? 1 : 0, es, 0).total;
      if (!decode && dt == ONE_DTYPE_BF16 && a.nv == 16 && 2 * (smem2 + 1024) <= 227 * 1024 &&
          (T + kAttnTok - 1) / kAttnTok > num_sms()) {
        a.minb = 2;
        a.smem = smem2;
      }
      if (a.smem > 220 * 1024) return fail(ONE_ERR_UNSUPPORTED, "attention/router weights exceed shared memory (%zu B)", a.smem);
      if (moe && (HH % 8 || D % 8 || (c.r * HH) % 8 || Dh % 8))
        return fail(ONE_ERR_UNSUPPORTED, "router shapes: H*H, D and head_dim must be multiples of 8");
      RowAttnParams& q = a.ra;
      memset(&q, 0, sizeof(q));
      q.T = T; q.H = H; q.Dh = Dh; q.r = c.r; q.E = c.num_experts; q.k = c.top_k; q.use_moe = moe ? 1 : 0;
      q.seq_len = decode ? 0 : seq_len;
      q.counters = counters;
      q.inv_freq = e->inv_freq;
      q.proj = B_(e->b.proj);
      q.attn_scale = 1.0f / sqrtf((float)Dh);
      q.wq = LW(ONE_W_LINQ_W); q.bq = LW(ONE_W_LINQ_B);
      q.wk = LW(ONE_W_LINK_W); q.bk = LW(ONE_W_LINK_B);
      q.wv = LW(ONE_W_LINV_W); q.bv = LW(ONE_W_LINV_B);
      q.o = moe ? nullptr : B_(e->b.o);
      if (moe) {
        const int k = c.top_k;
        int* ridx = e->at<int>(e->b.ridx);
        MoeRouter& r0 = q.rt[0];
        r0.gate_w = LW(ONE_W_HX_GATE); r0.experts = LW(ONE_W_HX_EXPERTS); r0.bias2 = LW(ONE_W_HX_BIAS2);
        r0.in = HH; r0.comb = B_(e->b.comb_hx); r0.idx_out = ridx;
        MoeRouter& r1 = q.rt[1];
        r1.gate_w = LW(ONE_W_X_GATE); r1.experts = LW(ONE_W_X_EXPERTS); r1.bias2 = LW(ONE_W_X_BIAS2);
        r1.in = HH; r1.comb = B_(e->b.comb_x); r1.idx_out = ridx + (size_t)T * k;
        MoeRouter& r2 = q.rt[2];
        r2.gate_w = nullptr; r2.glog = B_(e->b.gcx); r2.experts = LW(ONE_W_CX_EXPERTS); r2.bias2 = LW(ONE_W_CX_BIAS2);
        r2.x = B_(e->b.cxc[cur]); r2.ldx = D; r2.in = D; r2.comb = B_(e->b.comb_cx); r2.idx_out = ridx + (size_t)2 * T * k;
      }
      if (moe) q.tie = topk_tie_selection(c.num_experts, std::min(c.top_k, c.num_experts));
      q.err = err;
      plan.push_back(a);
    }
    // ---- gemm C: x_moe -> mean * clamp(.), the gate/up input. hx_moe and cx_moe are only
    // read by the next layer, so they run inside the gate/up launch (gemm D) instead of
    // lengthening this one (cx_moe has K = D, x_moe K = H*H).
    {
      ProbSpec ps[1];
      ps[0].kind = EPI_XMOE; ps[0].W = LW(ONE_W_X_W); ps[0].Nw = D; ps[0].K = HH;
      ps[0].X = moe ? B_(e->b.comb_x) : B_(e->b.o); ps[0].ldx = HH; ps[0].bias = LW(ONE_W_X_B);
      ps[0].out = B_(e->b.out0); ps[0].ldo = D; ps[0].aux = B_(e->b.mean); ps[0].lda = D;
      Launch g;
      int rc = plan_gemm(g, ps, 1, T, dt, err);
      if (rc) return rc;
      plan.push_back(g);
    }
    // ---- gemm D: gate/up | hx_moe -> hx + clamp(.) | cx_moe -> cx' and its clamp
    {
      ProbSpec ps[3];
      ps[0].kind = EPI_GELU_UP; ps[0].W = LW(ONE_W_GATE_UP); ps[0].Nw = 2 * I; ps[0].K = D;
      ps[0].X = B_(e->b.out0); ps[0].ldx = D; ps[0].bias = c.mlp_bias ? LW(ONE_W_GATE_UP_B) : nullptr;
      ps[0].out = B_(e->b.act); ps[0].ldo = I;
      ps[1].kind = EPI_HXPRE; ps[1].W = LW(ONE_W_HX_W); ps[1].Nw = D; ps[1].K = HH;
      ps[1].X = moe ? B_(e->b.comb_hx) : B_(e->b.o); ps[1].ldx = HH; ps[1].bias = LW(ONE_W_HX_B);
      ps[1].out = B_(e->b.hx_pre); ps[1].ldo = D; ps[1].aux = B_(e->b.hx); ps[1].lda = D;
      ps[2].kind = EPI_CX; ps[2].W = LW(ONE_W_CX_W); ps[2].Nw = D; ps[2].K = D;
      ps[2].X = moe ? B_(e->b.comb_cx) : B_(e->b.cx[cur]); ps[2].ldx = D; ps[2].bias = LW(ONE_W_CX_B);
      ps[2].out = B_(e->b.cx[nxt]); ps[2].ldo = D; ps[2].out2 = B_(e->b.cxc[nxt]); ps[2].ldo2 = D;
      Launch g;
      int rc = plan_gemm(g, ps, 3, T, dt, err);
      if (rc) return rc;
      plan.push_back(g);
    }
    // ---- gemm E: down, split-K partials
    {
      ProbSpec ps[1];
      ps[0].kind = EPI_PARTIAL; ps[0].W = LW(ONE_W_DOWN); ps[0].Nw = D; ps[0].K = I;
      ps[0].X = B_(e->b.act); ps[0].ldx = I; ps[0].ws = e->at<float>(e->b.ws); ps[0].ldw = D;
      ps[0].max_splits = std::max(1, std::min(kMaxSplits, e->b.ws_rows / std::max(T, 1)));
      Launch g;
      int rc = plan_gemm(g, ps, 1, T, dt, err);
      if (rc) return rc;
      GemmProblem& P = g.g.prob[0];
      if (g.kind == L_GEMM_TC && g.persist && P.splits == 1) {
        // unsplit (prompt ingestion): the epilogue adds the down bias and the residual out0
        // in place, so the next row_pre reads one bf16 row instead of an fp32 partial
        P.kind = EPI_RESID;
        P.bias = c.mlp_bias ? LW(ONE_W_DOWN_B) : nullptr;
        P.aux = B_(e->b.out0);
        P.lda = D;
        P.out = B_(e->b.out0);
        P.ldo = D;
      }
      plan.push_back(g);
    }
  }
  return ONE_OK;
}

// Final stage after the layers: finish the last layer, lhs_norm, up_scaler, model norm,
// lm_head (+argmax). Rows of the lm_head input: all T, or the last position of each
// sequence (prefill without full logits).
static int build_final(one_engine* e, std::vector<Launch>& plan, int T, int batch, int seq_len, bool last_only,
                       void* logits, bool advance, int* next_ids) {
  const one_config& c = e->c;
  const int D = c.transformer_dim, Hd = c.hidden_size;
  const int dt = c.dtype;
  const int nv = (D / 8 + 31) / 32;
  DevErr* err = e->at<DevErr>(e->b.err);
  auto B_ = [&](size_t off) { return e->at<void>(off); };
  const int L = c.num_hidden_layers;
  // splits of the last down_proj
  int splits = 1;
  for (auto it = plan.rbegin(); it != plan.rend(); ++it)
    if (it->kind == L_GEMM_TC || it->kind == L_GEMM_SIMT) {
      const GemmProblem& P = it->kind == L_GEMM_TC ? it->g.prob[0] : it->sg.prob[0];
      if (P.kind == EPI_PARTIAL) splits = P.splits;
      if (P.kind == EPI_RESID) splits = 0;
      break;
    }
  Launch rp;
  rp.dtype = dt;
  rp.nv = nv;
  row_pre_shape(rp, D, T, advance);
  RowPreParams& p = rp.rp;
  memset(&p, 0, sizeof(p));
  p.T = T;
  p.D = D;
  p.mode = PRE_FINAL;
  p.ws = e->at<float>(e->b.ws);
  p.splits = splits;
  p.out0 = B_(e->b.out0);
  p.prev_norm_w = e->L(L - 1, ONE_W_NORM_W);
  p.prev_norm_b = e->L(L - 1, ONE_W_NORM_B);
  if (c.mlp_bias) p.down_b = e->L(L - 1, ONE_W_DOWN_B);
  p.hx_pre = B_(e->b.hx_pre);
  p.hx = B_(e->b.hx);
  p.h = B_(e->b.h);
  p.lhs_w = e->gw[ONE_G_LHS_W];
  p.lhs_b = e->gw[ONE_G_LHS_B];
  p.hf = B_(e->b.hf);
  p.lhs_eps = c.rms_norm_eps;
  p.err = err;
  plan.push_back(rp);
  {
    ProbSpec ps[1];
    ps[0].W = e->gw[ONE_G_UP_W]; ps[0].Nw = Hd; ps[0].K = D; ps[0].X = B_(e->b.hf); ps[0].ldx = D;
    ps[0].bias = e->gw[ONE_G_UP_B]; ps[0].out = B_(e->b.u); ps[0].ldo = Hd;
    Launch g;
    int rc = plan_gemm(g, ps, 1, T, dt, err);
    if (rc) return rc;
    plan.push_back(g);
  }
  const int Tl = last_only ? batch : T;
  {
    Launch n;
    n.kind = L_ROW_NORM;
    n.dtype = dt;
    n.nv = (Hd / 8 + 31) / 32;
    n.block = 256;
    n.grid = (Tl + 7) / 8;
    n.rn = RowNormParams{Tl, Hd, B_(e->b.u), B_(e->b.hn), e->gw[ONE_G_NORM_W], e->gw[ONE_G_NORM_B], c.rms_norm_eps,
                         advance ? e->at<int>(e->b.counters) : nullptr, last_only ? seq_len : 1, last_only ? seq_len - 1 : 0};
    plan.push_back(n);
  }
  auto a16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
  if (dt == ONE_DTYPE_BF16 && Hd % 8 == 0 && a16(e->gw[ONE_G_LM_HEAD]) && a16(B_(e->b.hn))) {
    // lm_head + argmax with the tokens as the MMA's M rows (lm_head_argmax_kernel)
    Launch g;
    g.kind = L_LM_HEAD;
    g.dtype = dt;
    LmParams& q = g.lm;
    memset(&q, 0, sizeof(q));
    int rc = make_map(&q.tmx, B_(e->b.hn), Tl, Hd, Hd, 128);
    if (rc) return rc;
    rc = make_map(&q.tmw, e->gw[ONE_G_LM_HEAD], c.vocab_size, Hd, Hd, kLmBN);
    if (rc) return rc;
    q.T = Tl; q.V = c.vocab_size; q.K = Hd;
    q.t_tiles = (Tl + 127) / 128;
    q.logits = reinterpret_cast<__nv_bfloat16*>(logits);
    q.ldo = c.vocab_size;
    q.best = e->at<unsigned long long>(e->b.best);
    q.err = err;
    g.block = LmCfg::kThreads;
    g.smem = LmCfg::kSmem;
    g.grid = ((c.vocab_size + kLmBN - 1) / kLmBN) * ((q.t_tiles + kLmTT - 1) / kLmTT);
    plan.push_back(g);
  } else {
    ProbSpec ps[1];
    ps[0].kind = EPI_ARGMAX; ps[0].W = e->gw[ONE_G_LM_HEAD]; ps[0].Nw = c.vocab_size; ps[0].K = Hd;
    ps[0].X = B_(e->b.hn); ps[0].ldx = Hd; ps[0].out = logits; ps[0].ldo = c.vocab_size;
    ps[0].best = e->at<unsigned long long>(e->b.best);
    Launch g;
    int rc = plan_gemm(g, ps, 1, Tl, dt, err);
    if (rc) return rc;
    plan.push_back(g);
  }
  if (next_ids) {
    Launch n;
    n.kind = L_NEXT_IDS;
    n.block = 256;
    n.grid = (Tl + 255) / 256;
    n.ni = NextIdsParams{e->at<unsigned long long>(e->b.best), next_ids, Tl};
    plan.push_back(n);
  }
  return ONE_OK;
}

// after build_layers: propagate each down_proj split count to the row_pre that reads it
static void link_splits(std::vector<Launch>& plan) {
  int splits = 1;
  for (auto& L : plan) {
    if (L.kind == L_GEMM_TC || L.kind == L_GEMM_SIMT) {
      const GemmProblem& P = L.kind == L_GEMM_TC ? L.g.prob[0] : L.sg.prob[0];
      if (P.kind == EPI_PARTIAL) splits = P.splits;
      if (P.kind == EPI_RESID) splits = 0;
    } else if (L.kind == L_ROW_PRE || L.kind == L_ROW_PRE_W) {
      L.rp.splits = splits;
    }
  }
}

static int run_plan(const std::vector<Launch>& plan, cudaStream_t st) {
  for (const Launch& L : plan) {
    int rc = run(L, st);
    if (rc) return rc;
  }
  return ONE_OK;
}

extern "C" int one_engine_prefill(one_engine* e, const int32_t* ids, int32_t batch, int32_t seq_len,
                                  const float* prompt_div, int32_t logits_mode, void* logits, void* stream) {
  if (!e || !ids || !prompt_div || batch < 1 || seq_len < 1) return fail(ONE_ERR_INVALID, "bad prefill arguments");
  if (batch > e->max_batch) return fail(ONE_ERR_INVALID, "batch %d > max_batch %d", batch, e->max_batch);
  const long T = (long)batch * seq_len;
  if (T > e->max_tokens) return fail(ONE_ERR_INVALID, "batch*seq_len %ld > max_tokens %d", T, e->max_tokens);
  if (logits_mode && !logits) return fail(ONE_ERR_INVALID, "logits buffer required");
  cudaStream_t st = (cudaStream_t)stream;
  std::vector<Launch> plan;
  int rc = build_layers(e, plan, (int)T, false, seq_len, batch, ids, false, prompt_div);
  if (rc) return rc;
  link_splits(plan);
  rc = build_final(e, plan, (int)T, batch, seq_len, logits_mode != 2, logits_mode ? logits : nullptr, false, nullptr);
  if (rc) return rc;
  // lm_head argmax accumulates into `best`: clear it first
  CK(cudaMemsetAsync(e->ws + e->b.best, 0, (size_t)std::max(e->max_tokens, e->max_batch) * 8, st));
  rc = run_plan(plan, st);
  if (rc) return rc;
  Launch a;
  a.kind = L_ADVANCE;
  a.ad = AdvanceParams{e->at<int>(e->b.counters), seq_len, 0, 0, 0, 0};
  return run(a, st);
}

static int build_step(one_engine* e, std::vector<Launch>& plan, int batch, const int* ids, void* logits, int* next_ids) {
  int rc = build_layers(e, plan, batch, true, 0, batch, ids, ids == nullptr, nullptr);
  if (rc) return rc;
  link_splits(plan);
  return build_final(e, plan, batch, batch, 1, false, logits, true, next_ids);
}

extern "C" int one_engine_step(one_engine* e, int32_t batch, const int32_t* ids, void* logits, int32_t* next_ids,
                               void* stream) {
  if (!e || batch < 1 || batch > e->max_batch) return fail(ONE_ERR_INVALID, "bad batch");
  if (!e->use_graphs) {
    std::vector<Launch> plan;
    int rc = build_step(e, plan, batch, ids, logits, next_ids);
    if (rc) return rc;
    return run_plan(plan, (cudaStream_t)stream);
  }
  for (auto& sg : e->step_graphs)
    if (sg.batch == batch && sg.ids == ids && sg.logits == logits && sg.next_ids == next_ids) {
      CK(cudaGraphLaunch(sg.x, (cudaStream_t)stream));
      return ONE_OK;
    }
  std::vector<Launch> plan;
  int rc = build_step(e, plan, batch, ids, logits, next_ids);
  if (rc) return rc;
  one_engine::StepGraph sg{batch, ids, logits, next_ids, nullptr, nullptr};
  rc = capture_plan(e, plan, 1, &sg.g, &sg.x);
  if (rc) return rc;
  if (e->step_graphs.size() >= 8) {
    cudaGraphExecDestroy(e->step_graphs.front().x);
    cudaGraphDestroy(e->step_graphs.front().g);
    e->step_graphs.erase(e->step_graphs.begin());
  }
  e->step_graphs.push_back(sg);
  CK(cudaGraphLaunch(sg.x, (cudaStream_t)stream));
  return ONE_OK;
}

extern "C" int32_t one_engine_prefill_launches(one_engine* e, int32_t batch, int32_t seq_len, int32_t logits_mode) {
  if (!e || batch < 1 || seq_len < 1) return -1;
  std::vector<Launch> plan;
  if (build_layers(e, plan, batch * seq_len, false, seq_len, batch, nullptr, false, nullptr)) return -1;
  link_splits(plan);
  int32_t dummy = 0;
  if (build_final(e, plan, batch * seq_len, batch, seq_len, logits_mode != 2, logits_mode ? &dummy : nullptr, false,
                  nullptr))
    return -1;
  return (int32_t)plan.size() + 1;  // + the counter update
}

extern "C" int32_t one_engine_step_launches(one_engine* e, int32_t batch) {
  if (!e) return -1;
  std::vector<Launch> plan;
  if (build_step(e, plan, batch, nullptr, nullptr, nullptr)) return -1;
  return (int32_t)plan.size();
}

extern "C" int one_engine_capture(one_engine* e, int32_t batch, int32_t steps, void* stream) {
  if (!e || batch < 1 || batch > e->max_batch || steps < 1) return fail(ONE_ERR_INVALID, "bad capture arguments");
  std::vector<Launch> plan;
  int rc = build_step(e, plan, batch, nullptr, nullptr, nullptr);
  if (rc) return rc;
  (void)stream;
  if (e->graph) {
    cudaGraphExecDestroy(e->graph);
    e->graph = nullptr;
  }
  if (e->graph_def) {
    cudaGraphDestroy(e->graph_def);
    e->graph_def = nullptr;
  }
  return capture_plan(e, plan, steps, &e->graph_def, &e->graph);
}

extern "C" int one_engine_replay(one_engine* e, void* stream) {
  if (!e || !e->graph) return fail(ONE_ERR_INVALID, "no captured graph");
  CK(cudaGraphLaunch(e->graph, (cudaStream_t)stream));
  return ONE_OK;
}

extern "C" void* one_engine_buffer(one_engine* e, const char* name) {
  if (!e || !name) return nullptr;
  const int L = e->c.num_hidden_layers;
  if (!strcmp(name, "state")) return e->ws + e->b.state;
  if (!strcmp(name, "counters")) return e->ws + e->b.counters;
  if (!strcmp(name, "history")) return e->ws + e->b.hist;
  if (!strcmp(name, "hx")) return e->ws + e->b.hx;
  if (!strcmp(name, "cx")) return e->ws + e->b.cx[L & 1];
  if (!strcmp(name, "router_idx")) return e->ws + e->b.ridx;
  if (!strcmp(name, "best")) return e->ws + e->b.best;
  if (!strcmp(name, "ids_out")) return e->ws + e->b.ids_out;
  if (!strcmp(name, "h")) return e->ws + e->b.h;
  return nullptr;
}

extern "C" int one_engine_error(one_engine* e, int32_t* code, int32_t* where) {
  if (!e) return fail(ONE_ERR_INVALID, "null engine");
  DevErr h{0, 0};
  CK(cudaMemcpy(&h, e->ws + e->b.err, sizeof(h), cudaMemcpyDeviceToHost));
  if (code) *code = h.code;
  if (where) *where = h.where;
  return h.code != 0;
}

// Time every launch of a decode step separately: each launch runs `reps` times back to
// back between two CUDA events on `stream`; us_out[i] is the mean duration of launch i
// (warm caches). Returns the number of launches (<= n) or -1.
extern "C" int32_t one_engine_profile_step(one_engine* e, int32_t batch, int32_t reps, float* us_out, int32_t n,
                                           void* stream) {
  if (!e || batch < 1 || batch > e->max_batch || reps < 1 || !us_out) return -1;
  std::vector<Launch> plan;
  if (build_step(e, plan, batch, nullptr, nullptr, nullptr)) return -1;
  cudaStream_t st = (cudaStream_t)stream;
  cudaEvent_t a, b;
  if (cudaEventCreate(&a) != cudaSuccess || cudaEventCreate(&b) != cudaSuccess) return -1;
  const int m = std::min<int>(n, (int)plan.size());
  for (int i = 0; i < (int)plan.size(); ++i) {
    if (i < m) cudaEventRecord(a, st);
    for (int r = 0; r < (i < m ? reps : 1); ++r)
      if (run(plan[i], st)) return -1;
    if (i < m) {
      cudaEventRecord(b, st);
      cudaEventSynchronize(b);
      float ms = 0.f;
      cudaEventElapsedTime(&ms, a, b);
      us_out[i] = 1000.f * ms / reps;
    }
  }
  cudaEventDestroy(a);
  cudaEventDestroy(b);
  return m;
}

#include "capi_ops.cuh"
