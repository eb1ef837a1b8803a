// extern "C" standalone operators (one_b200.h, "standalone ops"). Included once, at the
// end of engine.cu, so they share its GEMM planner and launch helpers.
#pragma once

template <typename T>
__global__ void clamp_copy_kernel(const T* x, T* y, long n, float lim) {
  pdl_wait();
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) st<T>(y + i, fminf(fmaxf(ld<T>(x + i), -lim), lim));
}

// x.clamp(-1e4, 1e4) of a bf16 tensor (one/linear_moe.py:53), 16 bytes per thread per
// iteration over a grid of a few CTAs per SM: the bound is bf16(1e4) = 9984, and each packed
// min / max is exact, so the values equal clamp_copy_kernel's. n8 = elements / 8.
__global__ void clamp_copy_bf16x8_kernel(const uint4* x, uint4* y, long n8) {
  pdl_wait();
  const uint32_t hi = 0x461c461cu, lo = 0xc61cc61cu;  // +-9984
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n8; i += (long)gridDim.x * blockDim.x) {
    const uint4 v = x[i];
    y[i] = make_uint4(bf2_min(bf2_max(v.x, lo), hi), bf2_min(bf2_max(v.y, lo), hi), bf2_min(bf2_max(v.z, lo), hi),
                      bf2_min(bf2_max(v.w, lo), hi));
  }
}

static size_t align1k(size_t x) { return (x + 1023) & ~size_t(1023); }

extern "C" size_t one_linear_moe_workspace_bytes(int32_t n, int32_t fin, int32_t r, int32_t dtype) {
  const size_t es = dtype == ONE_DTYPE_F32 ? 4 : 2;
  return align1k((size_t)n * fin * es) * 2 + align1k((size_t)n * r * es) + 1024;
}

static int router_launch(const MoeRouter& R, int n, int r, int E, int k, int dtype, cudaStream_t st) {
  Launch L;
  const int rc = plan_router(L, R, n, r, E, k, dtype);
  return rc ? rc : run(L, st);
}

extern "C" int one_linear_moe(const void* x, int32_t n, int32_t fin, int32_t fout, const void* weight, const void* bias,
                              const void* gate_w, const void* experts, const void* bias2, int32_t num_experts, int32_t r,
                              int32_t top_k, int32_t dtype, void* out, int32_t* idx_out, void* workspace,
                              size_t workspace_bytes, void* stream) {
  if (!x || !weight || !gate_w || !experts || !bias2 || !out || !workspace) return fail(ONE_ERR_INVALID, "null argument");
  if (n < 1 || fin < 1 || fout < 1 || r < 1 || top_k < 1) return fail(ONE_ERR_INVALID, "sizes must be positive");
  if (num_experts < 1 || num_experts > kMaxExperts) return fail(ONE_ERR_UNSUPPORTED, "1..%d experts", kMaxExperts);
  if (fin > 4096) return fail(ONE_ERR_UNSUPPORTED, "in_features <= 4096");
  if (workspace_bytes < one_linear_moe_workspace_bytes(n, fin, r, dtype)) return fail(ONE_ERR_INVALID, "workspace too small");
  int rc = set_kernel_attrs();
  if (rc) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  const size_t es = dtype == ONE_DTYPE_F32 ? 4 : 2;
  uint8_t* ws = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(workspace) + 1023) & ~uintptr_t(1023));
  void* xc = ws;
  void* comb = ws + align1k((size_t)n * fin * es);
  void* glog = ws + 2 * align1k((size_t)n * fin * es);
  // x.clamp(-1e4, 1e4) (one/linear_moe.py:53)
  const long total = (long)n * fin;
  cudaError_t ce;
  if (dtype == ONE_DTYPE_BF16 && total % 8 == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0) {
    const long n8 = total / 8;
    const long blocks = std::min<long>((n8 + 255) / 256, (long)num_sms() * 8);
    ce = launch_k(clamp_copy_bf16x8_kernel, dim3((unsigned)blocks), dim3(256), 0, st, (const uint4*)x, (uint4*)xc, n8);
  } else {
    ce = dtype == ONE_DTYPE_BF16
             ? launch_k(clamp_copy_kernel<__nv_bfloat16>, dim3((total + 255) / 256), dim3(256), 0, st,
                        (const __nv_bfloat16*)x, (__nv_bfloat16*)xc, total, 1e4f)
             : launch_k(clamp_copy_kernel<float>, dim3((total + 255) / 256), dim3(256), 0, st, (const float*)x,
                        (float*)xc, total, 1e4f);
  }
  if (ce != cudaSuccess) return fail(ONE_ERR_CUDA, "clamp launch: %s", cudaGetErrorString(ce));
  // gate logits (:56)
  Launch g;
  ProbSpec ps;
  ps.W = gate_w; ps.Nw = r; ps.K = fin; ps.X = xc; ps.ldx = fin; ps.out = glog; ps.ldo = r;
  rc = plan_gemm(g, &ps, 1, n, dtype, nullptr);
  if (rc) return rc;
  rc = run(g, st);
  if (rc) return rc;
  // router + combine (:59-90)
  MoeRouter R;
  memset(&R, 0, sizeof(R));
  R.glog = glog; R.experts = experts; R.bias2 = bias2; R.x = xc; R.ldx = fin; R.in = fin; R.comb = comb; R.idx_out = idx_out;
  rc = router_launch(R, n, r, num_experts, top_k, dtype, st);
  if (rc) return rc;
  // shared Linear (:93)
  ProbSpec p2;
  p2.W = weight; p2.Nw = fout; p2.K = fin; p2.X = comb; p2.ldx = fin; p2.bias = bias; p2.out = out; p2.ldo = fout;
  rc = plan_gemm(g, &p2, 1, n, dtype, nullptr);
  if (rc) return rc;
  return run(g, st);
}

extern "C" int one_moe_routing(const void* x, int32_t n, int32_t fin, const void* gate_logits, const void* experts,
                               const void* bias2, int32_t num_experts, int32_t r, int32_t top_k, int32_t dtype, void* comb,
                               int32_t* idx_out, void* stream) {
  if (!x || !gate_logits || !experts || !bias2 || !comb) return fail(ONE_ERR_INVALID, "null argument");
  if (n < 1 || fin < 1 || fin > 4096 || r < 1 || top_k < 1 || num_experts < 1 || num_experts > kMaxExperts)
    return fail(ONE_ERR_INVALID, "bad sizes");
  int rc = set_kernel_attrs();
  if (rc) return rc;
  MoeRouter R;
  memset(&R, 0, sizeof(R));
  R.glog = gate_logits; R.experts = experts; R.bias2 = bias2; R.x = x; R.ldx = fin; R.in = fin; R.comb = comb; R.idx_out = idx_out;
  return router_launch(R, n, r, num_experts, top_k, dtype, (cudaStream_t)stream);
}

extern "C" int one_rotary_embedding(const int64_t* position_ids, int32_t batch, int32_t seq, const float* inv_freq,
                                    int32_t dim, int32_t dtype, void* cos_out, void* sin_out, void* stream) {
  if (!position_ids || !inv_freq || !cos_out || !sin_out || batch < 1 || seq < 1 || dim < 2 || dim % 2)
    return fail(ONE_ERR_INVALID, "bad rotary arguments");
  const int n = batch * seq;
  const long total = (long)n * (dim / 2);
  cudaStream_t st = (cudaStream_t)stream;
  cudaError_t e = dtype == ONE_DTYPE_BF16
                      ? launch_k(rotary_kernel<__nv_bfloat16>, dim3((total + 255) / 256), dim3(256), 0, st, position_ids,
                                 n, inv_freq, dim, (__nv_bfloat16*)cos_out, (__nv_bfloat16*)sin_out)
                      : launch_k(rotary_kernel<float>, dim3((total + 255) / 256), dim3(256), 0, st, position_ids, n,
                                 inv_freq, dim, (float*)cos_out, (float*)sin_out);
  if (e != cudaSuccess) return fail(ONE_ERR_CUDA, "rotary launch: %s", cudaGetErrorString(e));
  return ONE_OK;
}

extern "C" int one_cumsum_and_normalize(const void* x, int32_t b, int32_t s, int32_t d, int32_t seq_len, int32_t dtype,
                                        void* out, void* stream) {
  if (!x || !out || b < 1 || s < 1 || d < 1 || seq_len < 1) return fail(ONE_ERR_INVALID, "bad cumsum arguments");
  const long total = (long)b * d;
  cudaStream_t st = (cudaStream_t)stream;
  cudaError_t e = dtype == ONE_DTYPE_BF16
                      ? launch_k(cumsum_norm_kernel<__nv_bfloat16>, dim3((total + 255) / 256), dim3(256), 0, st,
                                 (const __nv_bfloat16*)x, b, s, d, seq_len, (__nv_bfloat16*)out)
                      : launch_k(cumsum_norm_kernel<float>, dim3((total + 255) / 256), dim3(256), 0, st, (const float*)x,
                                 b, s, d, seq_len, (float*)out);
  if (e != cudaSuccess) return fail(ONE_ERR_CUDA, "cumsum launch: %s", cudaGetErrorString(e));
  return ONE_OK;
}

extern "C" int one_combined_rope_attention(const void* single_x, const void* key, const void* value, const void* cosv,
                                           const void* sinv, int32_t cos_batch, const void* wq, const void* bq,
                                           const void* wk, const void* bk, const void* wv, const void* bv, int32_t b,
                                           int32_t h, int32_t t, int32_t dh, int32_t hout, int32_t dtype, void* out,
                                           void* stream) {
  if (!single_x || !key || !value || !cosv || !sinv || !wq || !wk || !wv || !out) return fail(ONE_ERR_INVALID, "null argument");
  if (b < 1 || h < 1 || t < 1 || dh < 2 || dh % 2 || hout < 1 || hout > 64) return fail(ONE_ERR_INVALID, "bad sizes");
  const long total = (long)b * h * t;
  cudaStream_t st = (cudaStream_t)stream;
  cudaError_t e;
  if (dtype == ONE_DTYPE_BF16) {
    using T = __nv_bfloat16;
    e = launch_k(combined_rope_attn_kernel<T>, dim3((total + 127) / 128), dim3(128), 0, st, (const T*)single_x,
                 (const T*)key, (const T*)value, (const T*)cosv, (const T*)sinv, (int)cos_batch, (const T*)wq, (const T*)bq,
                 (const T*)wk, (const T*)bk, (const T*)wv, (const T*)bv, (int)b, (int)h, (int)t, (int)dh, (int)hout, (T*)out);
  } else {
    using T = float;
    e = launch_k(combined_rope_attn_kernel<T>, dim3((total + 127) / 128), dim3(128), 0, st, (const T*)single_x,
                 (const T*)key, (const T*)value, (const T*)cosv, (const T*)sinv, (int)cos_batch, (const T*)wq, (const T*)bq,
                 (const T*)wk, (const T*)bk, (const T*)wv, (const T*)bv, (int)b, (int)h, (int)t, (int)dh, (int)hout, (T*)out);
  }
  if (e != cudaSuccess) return fail(ONE_ERR_CUDA, "combined attention launch: %s", cudaGetErrorString(e));
  return ONE_OK;
}

// ------------------------------------------------------------------ attention
// Error record shared by the standalone ops' kernels (bounded waits that ran out).
__device__ DevErr g_ops_err;
static DevErr* ops_err_ptr() {
  static std::mutex mu;
  static void* addr[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (!addr[dev] && cudaGetSymbolAddress(&addr[dev], g_ops_err) != cudaSuccess) addr[dev] = nullptr;
  return reinterpret_cast<DevErr*>(addr[dev]);
}

extern "C" int one_ops_error(int32_t* where, int32_t clear) {
  DevErr h{0, 0};
  CK(cudaDeviceSynchronize());
  CK(cudaMemcpyFromSymbol(&h, g_ops_err, sizeof(h)));
  if (clear) {
    const DevErr z{0, 0};
    CK(cudaMemcpyToSymbol(g_ops_err, &z, sizeof(z)));
  }
  if (where) *where = h.where;
  return h.code;
}

// bf16 3-D map over [bh][n][64] rows: box {64, 128, 1}, 128-byte swizzle, zero fill past n.
static int make_map_bhn(CUtensorMap* m, const void* ptr, int bh, int n) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(ONE_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  if (reinterpret_cast<uintptr_t>(ptr) & 15) return fail(ONE_ERR_INVALID, "attention operands must be 16-byte aligned");
  cuuint64_t dims[3] = {(cuuint64_t)kFaDh, (cuuint64_t)n, (cuuint64_t)bh};
  cuuint64_t strides[2] = {(cuuint64_t)kFaDh * 2, (cuuint64_t)n * kFaDh * 2};
  cuuint32_t box[3] = {(cuuint32_t)kFaDh, (cuuint32_t)kFaRows, 1};
  cuuint32_t es[3] = {1, 1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(ptr), dims, strides, box, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(ONE_ERR_CUDA, "cuTensorMapEncodeTiled (attention) failed (%d)", (int)r);
  return ONE_OK;
}

// The tensor-core kernel: bf16, head_dim 64, 16-byte aligned operands, and a positive
// scale (it takes the row max before scaling).
static bool attn_tc_eligible(const void* q, const void* k, const void* v, const void* out, int dh, float scale,
                             int dtype) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) |
                      reinterpret_cast<uintptr_t>(v) | reinterpret_cast<uintptr_t>(out);
  return dtype == ONE_DTYPE_BF16 && dh == kFaDh && (a & 15) == 0 && scale > 0.f && scale < 3.0e38f;
}

static int attn_launch(const void* q, const void* k, const void* v, int b, int h, int nq, int nk, int dh, int causal,
                       float scale, int dtype, void* out, cudaStream_t st) {
  cudaError_t e;
  if (attn_tc_eligible(q, k, v, out, dh, scale, dtype)) {
    int rc = set_kernel_attrs();
    if (rc) return rc;
    FaParams p;
    memset(&p, 0, sizeof(p));
    const int bh = b * h;
    if ((rc = make_map_bhn(&p.tq, q, bh, nq)) || (rc = make_map_bhn(&p.tk, k, bh, nk)) ||
        (rc = make_map_bhn(&p.tv, v, bh, nk)))
      return rc;
    p.out = (__nv_bfloat16*)out;
    p.nq = nq;
    p.nk = nk;
    p.causal = causal ? 1 : 0;
    p.scale_log2 = scale * 1.4426950408889634f;
    p.err = ops_err_ptr();
    static int resident = -1, regs = -1;
    if (resident < 0) {
      cudaFuncAttributes fa;
      CK(cudaFuncGetAttributes(&fa, flash_attn_tc_kernel));
      regs = fa.numRegs;
      CK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&resident, flash_attn_tc_kernel, kFaThreads, kFaSmem));
    }
    if (resident < 1) return fail(ONE_ERR_CUDA, "attention kernel does not fit on an SM (registers / shared memory)");
    // the kernel's setmaxnreg split assumes exactly this launch allocation; with fewer
    // registers the softmax warpgroups' increase could not be met
    if (regs != kFaRegsLaunch)
      return fail(ONE_ERR_UNSUPPORTED, "attention kernel built with %d registers per thread, expected %d", regs,
                  kFaRegsLaunch);
    const int pairs = (nq + kFaRows * kFaQTiles - 1) / (kFaRows * kFaQTiles);
    if (pairs > 65535) return fail(ONE_ERR_UNSUPPORTED, "attention: nq too large");
    e = launch_k(flash_attn_tc_kernel, dim3(bh, pairs), dim3(kFaThreads), kFaSmem, st, p);
  } else {
    if (dh > 64) return fail(ONE_ERR_UNSUPPORTED, "attention: head_dim <= 64 (tensor-core path: bf16, head_dim 64)");
    dim3 grid((nq + 63) / 64, b * h);
    e = dtype == ONE_DTYPE_BF16
            ? launch_k(attn_simt_kernel<__nv_bfloat16>, grid, dim3(64), 0, st, (const __nv_bfloat16*)q,
                       (const __nv_bfloat16*)k, (const __nv_bfloat16*)v, nq, nk, dh, causal, scale, (__nv_bfloat16*)out)
            : launch_k(attn_simt_kernel<float>, grid, dim3(64), 0, st, (const float*)q, (const float*)k,
                       (const float*)v, nq, nk, dh, causal, scale, (float*)out);
  }
  if (e != cudaSuccess) return fail(ONE_ERR_CUDA, "attention launch: %s", cudaGetErrorString(e));
  return ONE_OK;
}

extern "C" int one_flash_attention(const void* q, const void* k, const void* v, int32_t b, int32_t h, int32_t nq, int32_t nk,
                                   int32_t dh, int32_t causal, float scale, int32_t dtype, void* out, void* stream) {
  if (!q || !k || !v || !out || b < 1 || h < 1 || nq < 1 || nk < 1 || dh < 1)
    return fail(ONE_ERR_INVALID, "bad attention arguments");
  if ((long)b * h > 0x7fffffffL) return fail(ONE_ERR_UNSUPPORTED, "attention: b * h too large");
  return attn_launch(q, k, v, b, h, nq, nk, dh, causal, scale, dtype, out, (cudaStream_t)stream);
}

// x * cos + rotate_half(x) * sin for any dtype / even head_dim: one thread per element pair.
template <typename T>
__global__ void rope_qk_generic_kernel(const T* q, const T* k, const T* cosv, const T* sinv, int h, int n, int dh,
                                       long cs_bstride, long rows, T* qr, T* kr) {
  pdl_wait();
  const int half = dh / 2;
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows * 2 * half) return;
  const int e = (int)(i % half);
  long row = i / half;
  const bool is_k = row >= rows;
  if (is_k) row -= rows;
  const long bhi = row / n;
  const int pos = (int)(row - bhi * n);
  const long b = bhi / h;
  const T* x = (is_k ? k : q) + row * dh;
  const T* cs = cosv + b * cs_bstride + (long)pos * dh;
  const T* sn = sinv + b * cs_bstride + (long)pos * dh;
  const float x1 = ld<T>(x + e), x2 = ld<T>(x + half + e);
  T* y = (is_k ? kr : qr) + row * dh;
  st<T>(y + e, rnd<T>(x1 * ld<T>(cs + e)) + rnd<T>(-x2 * ld<T>(sn + e)));
  st<T>(y + half + e, rnd<T>(x2 * ld<T>(cs + half + e)) + rnd<T>(x1 * ld<T>(sn + half + e)));
}

extern "C" size_t one_rope_flash_attention_workspace_bytes(int32_t b, int32_t h, int32_t n, int32_t dh, int32_t dtype) {
  const size_t es = dtype == ONE_DTYPE_F32 ? 4 : 2;
  return 2 * align1k((size_t)b * h * n * dh * es) + 1024;
}

extern "C" int one_rope_flash_attention(const void* q, const void* k, const void* v, const void* cosv, const void* sinv,
                                        int32_t cos_batch, int32_t b, int32_t h, int32_t n, int32_t dh, int32_t causal,
                                        float scale, int32_t dtype, void* out, void* workspace, size_t workspace_bytes,
                                        void* stream) {
  if (!q || !k || !v || !cosv || !sinv || !out || !workspace || b < 1 || h < 1 || n < 1 || dh < 2 || (dh & 1))
    return fail(ONE_ERR_INVALID, "bad RoPE attention arguments");
  if (cos_batch != 1 && cos_batch != b) return fail(ONE_ERR_INVALID, "cos_batch must be 1 or b");
  if (workspace_bytes < one_rope_flash_attention_workspace_bytes(b, h, n, dh, dtype))
    return fail(ONE_ERR_INVALID, "workspace too small");
  cudaStream_t st = (cudaStream_t)stream;
  const size_t es = dtype == ONE_DTYPE_F32 ? 4 : 2;
  uint8_t* ws = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(workspace) + 1023) & ~uintptr_t(1023));
  void* qr = ws;
  void* kr = ws + align1k((size_t)b * h * n * dh * es);
  const long rows = (long)b * h * n;
  const long cs_bstride = cos_batch == 1 ? 0 : (long)n * dh;
  cudaError_t e;
  const uintptr_t al = reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) |
                       reinterpret_cast<uintptr_t>(cosv) | reinterpret_cast<uintptr_t>(sinv);
  if (dtype == ONE_DTYPE_BF16 && dh == 64 && (al & 15) == 0) {
    const long threads = rows * 8;
    e = launch_k(rope_qk_kernel, dim3((unsigned)((threads + 255) / 256)), dim3(256), 0, st, (const __nv_bfloat16*)q,
                 (const __nv_bfloat16*)k, (const __nv_bfloat16*)cosv, (const __nv_bfloat16*)sinv, (int)h, (int)n,
                 cs_bstride, rows, (__nv_bfloat16*)qr, (__nv_bfloat16*)kr);
  } else {
    const long threads = rows * dh;
    const dim3 grid((unsigned)((threads + 255) / 256));
    e = dtype == ONE_DTYPE_BF16
            ? launch_k(rope_qk_generic_kernel<__nv_bfloat16>, grid, dim3(256), 0, st, (const __nv_bfloat16*)q,
                       (const __nv_bfloat16*)k, (const __nv_bfloat16*)cosv, (const __nv_bfloat16*)sinv, (int)h, (int)n,
                       (int)dh, cs_bstride, rows, (__nv_bfloat16*)qr, (__nv_bfloat16*)kr)
            : launch_k(rope_qk_generic_kernel<float>, grid, dim3(256), 0, st, (const float*)q, (const float*)k,
                       (const float*)cosv, (const float*)sinv, (int)h, (int)n, (int)dh, cs_bstride, rows, (float*)qr,
                       (float*)kr);
  }
  if (e != cudaSuccess) return fail(ONE_ERR_CUDA, "RoPE launch: %s", cudaGetErrorString(e));
  return attn_launch(qr, kr, v, b, h, n, n, dh, causal, scale, dtype, out, st);
}

// every bf16 dividend a (blockIdx.x * blockDim.x + threadIdx.x = its bit pattern) against
// divisors[blockIdx.y]
__global__ void selftest_division_kernel(const float* div, unsigned long long* mism) {
  const uint32_t bits = blockIdx.x * blockDim.x + threadIdx.x;
  if (bits >= 65536u) return;
  const float a = __uint_as_float(bits << 16), b = div[blockIdx.y];
  const float ref = a / b, got = div_rn_recip(a, b, 1.0f / b);
  const bool nan2 = isnan(ref) && isnan(got);
  const uint32_t r16 = pack_bf16x2(ref, ref) & 0xffffu, g16 = pack_bf16x2(got, got) & 0xffffu;
  if (!nan2 && __float_as_uint(ref) != __float_as_uint(got)) atomicAdd(&mism[0], 1ull);
  if (!nan2 && r16 != g16) atomicAdd(&mism[1], 1ull);
}

extern "C" int one_selftest_mean_division(const float* divisors, int32_t n, unsigned long long* mismatches,
                                          void* stream) {
  if (!divisors || !mismatches || n < 1 || n > 65535) return fail(ONE_ERR_INVALID, "bad self-test arguments");
  cudaStream_t st = (cudaStream_t)stream;
  CK(cudaMemsetAsync(mismatches, 0, 16, st));
  selftest_division_kernel<<<dim3(256, n), 256, 0, st>>>(divisors, mismatches);
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return fail(ONE_ERR_CUDA, "division self-test: %s", cudaGetErrorString(e));
  return ONE_OK;
}

extern "C" int one_sample_tokens(const void* logits, int32_t batch, int32_t vocab, int32_t ld, int32_t dtype,
                                 float temperature, int32_t top_k, float top_p, uint64_t seed, uint64_t offset,
                                 int32_t* out, void* stream) {
  if (!logits || !out) return fail(ONE_ERR_INVALID, "null argument");
  if (batch < 1 || vocab < 1 || ld < vocab) return fail(ONE_ERR_INVALID, "bad sizes");
  if (vocab > kSampMaxVocab) return fail(ONE_ERR_UNSUPPORTED, "vocabulary of at most %d entries", kSampMaxVocab);
  if (!(temperature > 0.0f)) return fail(ONE_ERR_INVALID, "temperature must be positive (do_sample=False is greedy)");
  if (top_k < 0 || !(top_p > 0.0f)) return fail(ONE_ERR_INVALID, "top_k >= 0 and top_p > 0");
  if (dtype != ONE_DTYPE_BF16 && dtype != ONE_DTYPE_F32) return fail(ONE_ERR_INVALID, "dtype");
  int rc = set_kernel_attrs();
  if (rc) return rc;
  SampleParams p{logits, batch, vocab, ld, dtype, temperature, top_k, top_p, (unsigned long long)seed,
                 (unsigned long long)offset, out};
  const cudaError_t e = launch_k(sample_kernel, dim3(batch), dim3(kSampThreads), (size_t)vocab * 4,
                                 (cudaStream_t)stream, p);
  if (e != cudaSuccess) return fail(ONE_ERR_CUDA, "sample launch: %s", cudaGetErrorString(e));
  return ONE_OK;
}
