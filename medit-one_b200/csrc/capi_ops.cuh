// extern "C" standalone operators (one_b200.h, "standalone ops"). Included once, at the
// end of engine.cu, so they share its GEMM planner and launch helpers.
#pragma once

template <typename T>
__global__ void clamp_copy_kernel(const T* x, T* y, long n, float lim) {
  pdl_wait();
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) st<T>(y + i, fminf(fmaxf(ld<T>(x + i), -lim), lim));
}

static size_t align1k(size_t x) { return (x + 1023) & ~size_t(1023); }

extern "C" size_t one_linear_moe_workspace_bytes(int32_t n, int32_t fin, int32_t r, int32_t dtype) {
  const size_t es = dtype == ONE_DTYPE_F32 ? 4 : 2;
  return align1k((size_t)n * fin * es) * 2 + align1k((size_t)n * r * es) + 1024;
}

static int router_launch(const MoeRouter& R, int n, int r, int E, int k, int dtype, cudaStream_t st) {
  const size_t smem = moe_router_smem_bytes(R.in, r);
  const int grid = std::min(n, num_sms() * 8);
  cudaError_t e = dtype == ONE_DTYPE_BF16
                      ? launch_k(moe_router_kernel<__nv_bfloat16>, dim3(grid), dim3(128), smem, st, R, n, r, E, k)
                      : launch_k(moe_router_kernel<float>, dim3(grid), dim3(128), smem, st, R, n, r, E, k);
  if (e != cudaSuccess) return fail(ONE_ERR_CUDA, "router launch: %s", cudaGetErrorString(e));
  return ONE_OK;
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
  cudaError_t ce = dtype == ONE_DTYPE_BF16
                       ? launch_k(clamp_copy_kernel<__nv_bfloat16>, dim3((total + 255) / 256), dim3(256), 0, st,
                                  (const __nv_bfloat16*)x, (__nv_bfloat16*)xc, total, 1e4f)
                       : launch_k(clamp_copy_kernel<float>, dim3((total + 255) / 256), dim3(256), 0, st, (const float*)x,
                                  (float*)xc, total, 1e4f);
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

extern "C" int one_flash_attention(const void* q, const void* k, const void* v, int32_t b, int32_t h, int32_t nq, int32_t nk,
                                   int32_t dh, int32_t causal, float scale, int32_t dtype, void* out, void* stream) {
  if (!q || !k || !v || !out || b < 1 || h < 1 || nq < 1 || nk < 1 || dh < 1 || dh > 64)
    return fail(ONE_ERR_INVALID, "bad attention arguments");
  cudaStream_t st = (cudaStream_t)stream;
  dim3 grid((nq + 63) / 64, b * h);
  cudaError_t e = dtype == ONE_DTYPE_BF16
                      ? launch_k(attn_simt_kernel<__nv_bfloat16>, grid, dim3(64), 0, st, (const __nv_bfloat16*)q,
                                 (const __nv_bfloat16*)k, (const __nv_bfloat16*)v, (int)nq, (int)nk, (int)dh, (int)causal,
                                 scale, (__nv_bfloat16*)out)
                      : launch_k(attn_simt_kernel<float>, grid, dim3(64), 0, st, (const float*)q, (const float*)k,
                                 (const float*)v, (int)nq, (int)nk, (int)dh, (int)causal, scale, (float*)out);
  if (e != cudaSuccess) return fail(ONE_ERR_CUDA, "attention launch: %s", cudaGetErrorString(e));
  return ONE_OK;
}
