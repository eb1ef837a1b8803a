// Per-token ("row") kernels of the decode / prefill step. Each restates a stretch of
// One.forward (one/modeling_one.py:325-590) or OneModel.forward (:727-803) that needs a
// whole hidden row: the RMSNorm chain between layers, the running-sum state, the
// feature attention and the three LinearMoE routers.
#pragma once

#include "common.cuh"
#include "topk.cuh"

namespace one {

// ------------------------------------------------------------------ RMSNorm over a warp row
// OneRMSNorm.forward (one/modeling_one.py:62-67): fp32 variance, x * rsqrt(var + eps),
// cast to the model dtype, times weight, plus bias (when the norm has one).
// The row lives in registers: lane owns 8-element chunks c = lane + 32 * j.
template <typename T, int NV>
ONE_DEVINL void warp_rmsnorm(float (&x)[NV][8], int nchunks, const T* w, const T* b, float eps, int D, float (&y)[NV][8]) {
  const int lane = threadIdx.x & 31;
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    if (lane + 32 * j < nchunks) {
#pragma unroll
      for (int e = 0; e < 8; ++e) ss += x[j][e] * x[j][e];
    }
  }
  ss = warp_sum(ss);
  const float r = 1.0f / sqrtf(ss / (float)D + eps);
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int c = lane + 32 * j;
    if (c < nchunks) {
      float wv[8], bv[8];
      load8(w + c * 8, wv);
      if (b) load8(b + c * 8, bv);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        float v = rnd<T>(wv[e] * rnd<T>(x[j][e] * r));
        if (b) v = rnd<T>(v + bv[e]);
        y[j][e] = v;
      }
    }
  }
}

template <typename T, int NV>
ONE_DEVINL void warp_load_row(const T* p, int nchunks, float (&x)[NV][8]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int j = 0; j < NV; ++j)
    if (lane + 32 * j < nchunks) load8(p + (lane + 32 * j) * 8, x[j]);
}
template <typename T, int NV>
ONE_DEVINL void warp_store_row(T* p, int nchunks, const float (&x)[NV][8]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int j = 0; j < NV; ++j)
    if (lane + 32 * j < nchunks) store8(p + (lane + 32 * j) * 8, x[j]);
}

// ------------------------------------------------------------------ layer entry
enum RowPreMode : int {
  PRE_FIRST = 0,  // layer 0: embed the token (:728), hx = 1, cx = embedding (:748-753)
  PRE_MID = 1,    // layer l > 0: finish layer l-1, then enter layer l
  PRE_FINAL = 2,  // after the last layer: finish it, then lhs_norm (:801)
};

struct RowPreParams {
  int T, D, vocab;
  int mode;
  int ids_from_best;      // PRE_FIRST: token = argmax key of the previous step, else ids[]
  int decode;             // update the running sum and write the mean (decode); prefill: scan later
  const int* ids;         // [T]
  unsigned long long* best;  // [T] argmax keys of the previous step (reset here)
  int* ids_out;           // [T] token fed this step (greedy)
  int* hist;              // [max_steps][T] generated tokens, or null
  int hist_cap;
  const int* counters;    // {pos, step}
  const void* emb;        // [V, D]
  const float* div;       // divisor per position (decode)
  int div_len;
  // previous layer's tail
  const float* ws;        // [splits][T][D] down_proj partials
  int splits;             // 0: out0 already holds out0 + down_proj(...) (EPI_RESID)
  const void* down_b;     // down_proj bias (mlp_bias) or null
  const void* out0;       // [T, D] mean * x_moe (the MLP input)
  const void* hx_pre;     // [T, D] hx + hx_moe, before norm
  const void* prev_norm_w;
  const void* prev_norm_b;
  // this layer
  const void* norm1_w;
  void* h;                // [T, D] residual stream (in/out)
  void* norm_x;           // [T, D]
  void* hx;               // [T, D]
  void* cx;               // [T, D]  (PRE_FIRST writes it)
  void* cxc;              // [T, D]  clamp(cx, +-1e4)
  float* S;               // [T, D] running sum of this layer (decode)
  void* mean;             // [T, D]
  const void* lhs_w;      // PRE_FINAL
  const void* lhs_b;
  void* hf;               // PRE_FINAL output [T, D]
  float lhs_eps;
  DevErr* err;
};

// Sum over the CTA: warp shuffle, then across warps through red[slot * 32 + warp].
template <int N>
ONE_DEVINL void block_sum(float (&v)[N], float* red, int slot) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
#pragma unroll
  for (int i = 0; i < N; ++i) {
    v[i] = warp_sum(v[i]);
    if (lane == 0) red[(slot + i) * 32 + warp] = v[i];
  }
  __syncthreads();
#pragma unroll
  for (int i = 0; i < N; ++i) {
    float s = 0.f;
    for (int w = 0; w < nw; ++w) s += red[(slot + i) * 32 + w];
    v[i] = s;
  }
}

// y = norm(x) for this thread's chunk, given the row's sum of squares.
template <typename T>
ONE_DEVINL void chunk_norm(const float* x, float ss, int D, float eps, const T* w, const T* b, int c, float* y) {
  const float r = 1.0f / sqrtf(ss / (float)D + eps);
  float wv[8], bv[8];
  load8(w + c * 8, wv);
  if (b) load8(b + c * 8, bv);
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    float v = rnd<T>(wv[e] * rnd<T>(x[e] * r));
    y[e] = b ? rnd<T>(v + bv[e]) : v;
  }
}

// chunk_norm with the weight / bias chunk already in registers (bv unused when has_b is false)
template <typename T>
ONE_DEVINL void chunk_norm_r(const float* x, float ss, int D, float eps, const float* wv, const float* bv, bool has_b,
                             float* y) {
  const float r = 1.0f / sqrtf(ss / (float)D + eps);
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    float v = rnd<T>(wv[e] * rnd<T>(x[e] * r));
    y[e] = has_b ? rnd<T>(v + bv[e]) : v;
  }
}

ONE_DEVINL float sumsq8(const float* x) {
  float s = 0.f;
#pragma unroll
  for (int e = 0; e < 8; ++e) s += x[e] * x[e];
  return s;
}

// One CTA per token; thread c owns elements [8c, 8c+8) of the D-wide rows. Every global
// load of the token is issued before the first reduction.
template <typename T>
__global__ void __launch_bounds__(128) row_pre_kernel(const RowPreParams p) {
  __shared__ float red[4 * 32];
  const int t = blockIdx.x;
  const int c = threadIdx.x;
  const int D = p.D;
  const bool act = c < D / 8;
  const size_t off = (size_t)t * D + (size_t)c * 8;
  float h[8], a[8], b[8];
  // weights (not written by any kernel of the step): before the dependency wait
  float w1[8], pw[8], pb[8], db[8];
  const bool mid = p.mode != PRE_FIRST;
  if (act) {
    // norm1 is absent in PRE_FINAL (the kernel returns before norm_x there)
    if (p.norm1_w) load8(reinterpret_cast<const T*>(p.norm1_w) + c * 8, w1);
    if (mid && p.prev_norm_w) {
      load8(reinterpret_cast<const T*>(p.prev_norm_w) + c * 8, pw);
      if (p.prev_norm_b) load8(reinterpret_cast<const T*>(p.prev_norm_b) + c * 8, pb);
      if (p.down_b) load8(reinterpret_cast<const T*>(p.down_b) + c * 8, db);
    }
  }
  pdl_launch_dependents();
  pdl_wait();

  if (p.mode == PRE_FIRST) {
    __shared__ int sid;
    if (threadIdx.x == 0) {
      int id = p.ids_from_best ? 0 : p.ids[t];
      if (p.ids_from_best) {
        const unsigned long long key = p.best[t];
        id = key ? (int)(0xFFFFFFFFu - (uint32_t)(key & 0xFFFFFFFFull)) : 0;
      }
      if (id < 0 || id >= p.vocab) {  // never gather outside the embedding table
        set_err(p.err, ERR_BAD_ARG, 100);
        id = 0;
      }
      // this step's lm_head argmax accumulates into best[t] again
      p.best[t] = 0ull;
      if (p.ids_out) p.ids_out[t] = id;
      if (p.hist) {
        const int step = p.counters[1];
        if (step < p.hist_cap) p.hist[(size_t)step * p.T + t] = id;
      }
      sid = id;
    }
    __syncthreads();
    if (act) {
      load8(reinterpret_cast<const T*>(p.emb) + (size_t)sid * D + c * 8, h);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        a[e] = 1.0f;
        b[e] = fminf(fmaxf(h[e], -1e4f), 1e4f);
      }
      store8(reinterpret_cast<T*>(p.hx) + off, a);
      store8(reinterpret_cast<T*>(p.cx) + off, h);
      store8(reinterpret_cast<T*>(p.cxc) + off, b);
    }
  }
  // the running-sum row of this layer (read-modify-write below), requested early
  float sr[8];
  if (p.decode && act && p.mode != PRE_FINAL) load8(p.S + off, sr);
  if (mid) {
    // finish the previous layer: out = norm(out0 + down_proj(...)) (:571-573), h += out (:793),
    // hx = norm(hx + hx_moe) (:563-564). The split-K partials are loaded eight at a time
    // before they are added, in split order.
    float hp[8];
    if (act) {
      float m[8];
      load8(reinterpret_cast<const T*>(p.out0) + off, a);
      load8(reinterpret_cast<const T*>(p.h) + off, h);
      load8(reinterpret_cast<const T*>(p.hx_pre) + off, hp);
      // splits == 0: the down_proj epilogue already stored out0 + down_proj(...) in out0
      for (int s0 = 0; s0 < p.splits; s0 += 8) {
        float v[8][8];
#pragma unroll
        for (int j = 0; j < 8; ++j)
          if (s0 + j < p.splits) load8(p.ws + (size_t)(s0 + j) * p.T * D + off, v[j]);
#pragma unroll
        for (int j = 0; j < 8; ++j)
          if (s0 + j < p.splits) {
#pragma unroll
            for (int e = 0; e < 8; ++e) m[e] = (s0 + j == 0) ? v[j][e] : m[e] + v[j][e];
          }
      }
      if (p.splits > 0) {
        if (p.down_b)
#pragma unroll
          for (int e = 0; e < 8; ++e) m[e] += db[e];
#pragma unroll
        for (int e = 0; e < 8; ++e) a[e] = rnd<T>(a[e] + rnd<T>(m[e]));
      }
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) a[e] = h[e] = hp[e] = 0.f;
    }
    float ss[2] = {sumsq8(a), sumsq8(hp)};
    block_sum<2>(ss, red, 0);
    if (act) {
      chunk_norm_r<T>(a, ss[0], D, 1e-6f, pw, pb, p.prev_norm_b != nullptr, b);
#pragma unroll
      for (int e = 0; e < 8; ++e) h[e] = rnd<T>(h[e] + b[e]);
      chunk_norm_r<T>(hp, ss[1], D, 1e-6f, pw, pb, p.prev_norm_b != nullptr, b);
      store8(reinterpret_cast<T*>(p.hx) + off, b);
      store8(reinterpret_cast<T*>(p.h) + off, h);
    }
    if (p.mode == PRE_FINAL) {
      float s3[1] = {act ? sumsq8(h) : 0.f};
      block_sum<1>(s3, red, 2);
      if (act) {
        chunk_norm<T>(h, s3[0], D, p.lhs_eps, reinterpret_cast<const T*>(p.lhs_w), reinterpret_cast<const T*>(p.lhs_b), c, a);
        store8(reinterpret_cast<T*>(p.hf) + off, a);
      }
      return;
    }
  }
  if (p.mode == PRE_FIRST && act) store8(reinterpret_cast<T*>(p.h) + off, h);
  // norm_x = norm1(h) (:340); OneRMSNorm(dim) keeps eps = 1e-6 and has no bias
  float s3[1] = {act ? sumsq8(h) : 0.f};
  block_sum<1>(s3, red, 3);
  if (!act) return;
  chunk_norm_r<T>(h, s3[0], D, 1e-6f, w1, w1, false, a);
  store8(reinterpret_cast<T*>(p.norm_x) + off, a);
  if (p.decode) {
    // running sum replaces cache.update + cumsum (:358-376); mean = sum / arange[-1] (:379-387)
    int pi = p.counters[0];
    if (pi >= p.div_len) {  // position beyond the divisor table the engine was built with
      if (threadIdx.x == 0) set_err(p.err, ERR_BAD_ARG, 101);
      pi = p.div_len - 1;
    }
    const float dv = p.div[pi];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      sr[e] += a[e];
      b[e] = rnd<T>(rnd<T>(sr[e]) / dv);
    }
    store8(p.S + off, sr);
    store8(reinterpret_cast<T*>(p.mean) + off, b);
  }
}

// Prompt-ingestion variant of row_pre_kernel (decode = 0): one warp per token, lane l owns
// the 8-element chunks l, l + 32, ... (NV of them), reductions by warp shuffles only (no CTA
// barrier). Same steps and rounding as row_pre_kernel; the row sums of squares are added in
// another order (fp32), as any reduction of the reference's norm may be.
// PRE_FIRST, one lane per token: the token id (fed back from the argmax, or given), checked
// against the vocabulary, recorded in ids_out / the history; clears the argmax slot.
ONE_DEVINL int first_token_id(const RowPreParams& p, int t) {
  int id = p.ids_from_best ? 0 : p.ids[t];
  if (p.ids_from_best) {
    const unsigned long long key = p.best[t];
    id = key ? (int)(0xFFFFFFFFu - (uint32_t)(key & 0xFFFFFFFFull)) : 0;
  }
  if (id < 0 || id >= p.vocab) {  // never gather outside the embedding table
    set_err(p.err, ERR_BAD_ARG, 100);
    id = 0;
  }
  p.best[t] = 0ull;
  if (p.ids_out) p.ids_out[t] = id;
  if (p.hist) {
    const int step = p.counters[1];
    if (step < p.hist_cap) p.hist[(size_t)step * p.T + t] = id;
  }
  return id;
}

template <typename T, int NV>
__global__ void __launch_bounds__(128, 3) row_pre_warp_kernel(const RowPreParams p) {
  const int lane = threadIdx.x & 31;
  const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  pdl_launch_dependents();
  pdl_wait();
  if (t >= p.T) return;
  const int D = p.D, nch = D / 8;
  const size_t row = (size_t)t * D;
  bool act[NV];
#pragma unroll
  for (int v = 0; v < NV; ++v) act[v] = lane + 32 * v < nch;
  float h[NV][8], a[NV][8], b[8];
  if (p.mode == PRE_FIRST) {
    int id = 0;
    if (lane == 0) id = first_token_id(p, t);
    id = __shfl_sync(0xffffffffu, id, 0);
#pragma unroll
    for (int v = 0; v < NV; ++v)
      if (act[v]) {
        const size_t off = row + (size_t)(lane + 32 * v) * 8;
        load8(reinterpret_cast<const T*>(p.emb) + (size_t)id * D + (lane + 32 * v) * 8, h[v]);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          a[v][e] = 1.0f;
          b[e] = fminf(fmaxf(h[v][e], -1e4f), 1e4f);
        }
        store8(reinterpret_cast<T*>(p.hx) + off, a[v]);
        store8(reinterpret_cast<T*>(p.cx) + off, h[v]);
        store8(reinterpret_cast<T*>(p.cxc) + off, b);
        store8(reinterpret_cast<T*>(p.h) + off, h[v]);
      }
  } else {
    // finish the previous layer (:571-573, :793, :563-564); split-K partials added in order
    // the first down_proj partial is requested with the other rows (one memory round trip when
    // there is a single split, as in prompt ingestion)
    float hp[NV][8], m[NV][8];
#pragma unroll
    for (int v = 0; v < NV; ++v)
      if (act[v]) {
        const size_t off = row + (size_t)(lane + 32 * v) * 8;
        load8(reinterpret_cast<const T*>(p.out0) + off, a[v]);
        load8(reinterpret_cast<const T*>(p.h) + off, h[v]);
        load8(reinterpret_cast<const T*>(p.hx_pre) + off, hp[v]);
        if (p.splits > 0) load8(p.ws + off, m[v]);
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) a[v][e] = h[v][e] = hp[v][e] = m[v][e] = 0.f;
      }
    for (int sp = 1; sp < p.splits; ++sp) {
      float w[NV][8];
#pragma unroll
      for (int v = 0; v < NV; ++v)
        if (act[v]) load8(p.ws + (size_t)sp * p.T * D + row + (size_t)(lane + 32 * v) * 8, w[v]);
#pragma unroll
      for (int v = 0; v < NV; ++v)
#pragma unroll
        for (int e = 0; e < 8; ++e) m[v][e] += w[v][e];
    }
    float ss0 = 0.f, ss1 = 0.f;
#pragma unroll
    for (int v = 0; v < NV; ++v)
      if (act[v]) {
        if (p.splits > 0) {  // splits == 0: out0 already holds out0 + down_proj(...)
          if (p.down_b) {
            float db[8];
            load8(reinterpret_cast<const T*>(p.down_b) + (lane + 32 * v) * 8, db);
#pragma unroll
            for (int e = 0; e < 8; ++e) m[v][e] += db[e];
          }
#pragma unroll
          for (int e = 0; e < 8; ++e) a[v][e] = rnd<T>(a[v][e] + rnd<T>(m[v][e]));
        }
        ss0 += sumsq8(a[v]);
        ss1 += sumsq8(hp[v]);
      }
    ss0 = warp_sum(ss0);
    ss1 = warp_sum(ss1);
#pragma unroll
    for (int v = 0; v < NV; ++v)
      if (act[v]) {
        const int c = lane + 32 * v;
        const size_t off = row + (size_t)c * 8;
        float pw[8], pb[8];
        load8(reinterpret_cast<const T*>(p.prev_norm_w) + c * 8, pw);
        if (p.prev_norm_b) load8(reinterpret_cast<const T*>(p.prev_norm_b) + c * 8, pb);
        chunk_norm_r<T>(a[v], ss0, D, 1e-6f, pw, pb, p.prev_norm_b != nullptr, b);
#pragma unroll
        for (int e = 0; e < 8; ++e) h[v][e] = rnd<T>(h[v][e] + b[e]);
        chunk_norm_r<T>(hp[v], ss1, D, 1e-6f, pw, pb, p.prev_norm_b != nullptr, b);
        store8(reinterpret_cast<T*>(p.hx) + off, b);
        store8(reinterpret_cast<T*>(p.h) + off, h[v]);
      }
    if (p.mode == PRE_FINAL) {
      float s3 = 0.f;
#pragma unroll
      for (int v = 0; v < NV; ++v)
        if (act[v]) s3 += sumsq8(h[v]);
      s3 = warp_sum(s3);
#pragma unroll
      for (int v = 0; v < NV; ++v)
        if (act[v]) {
          const int c = lane + 32 * v;
          chunk_norm<T>(h[v], s3, D, p.lhs_eps, reinterpret_cast<const T*>(p.lhs_w),
                        reinterpret_cast<const T*>(p.lhs_b), c, b);
          store8(reinterpret_cast<T*>(p.hf) + row + (size_t)c * 8, b);
        }
      return;
    }
  }
  // norm_x = norm1(h) (:340)
  float s3 = 0.f;
#pragma unroll
  for (int v = 0; v < NV; ++v)
    if (act[v]) s3 += sumsq8(h[v]);
  s3 = warp_sum(s3);
#pragma unroll
  for (int v = 0; v < NV; ++v)
    if (act[v]) {
      const int c = lane + 32 * v;
      float w1[8];
      load8(reinterpret_cast<const T*>(p.norm1_w) + c * 8, w1);
      chunk_norm_r<T>(h[v], s3, D, 1e-6f, w1, w1, false, b);
      store8(reinterpret_cast<T*>(p.norm_x) + row + (size_t)c * 8, b);
    }
}

// row_pre_warp_kernel for bf16 rows at the first layer (PRE_FIRST), and at the later layers
// and the final stage after an unsplit down_proj (splits == 0: out0 already holds
// out0 + down_proj(...)). The input rows stay packed bf16 in registers until each step
// unpacks the chunk it needs, so six CTAs (24 warps) fit an SM instead of three. Same steps,
// rounding and summation order as row_pre_warp_kernel: bit-identical.
ONE_DEVINL void unpack8(const uint4& u, float* v) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    v[2 * i] = bf2_lo(w[i]);
    v[2 * i + 1] = bf2_hi(w[i]);
  }
}

template <int NV>
__global__ void __launch_bounds__(128, NV <= 3 ? 6 : 5) row_pre_packed_kernel(const RowPreParams p) {
  using T = __nv_bfloat16;
  const int lane = threadIdx.x & 31;
  const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  pdl_launch_dependents();
  pdl_wait();
  if (t >= p.T) return;
  const int D = p.D, nch = D / 8;
  const size_t row = (size_t)t * D;
  const uint4 z = make_uint4(0, 0, 0, 0);
  uint4 uh[NV];
  if (p.mode == PRE_FIRST) {
    // embedding row (:335); hx = 1, cx = h, the LinearMoE-clamped cx (+-bf16(1e4) = +-9984:
    // the bf16 rounding of the fp32 clamp of a bf16 value)
    int id = 0;
    if (lane == 0) id = first_token_id(p, t);
    id = __shfl_sync(0xffffffffu, id, 0);
    const uint4 one = make_uint4(0x3f803f80u, 0x3f803f80u, 0x3f803f80u, 0x3f803f80u);
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      uh[v] = z;
      if (lane + 32 * v < nch) {
        const size_t off = row + (size_t)(lane + 32 * v) * 8;
        const uint4 e = *reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(p.emb) + (size_t)id * D + (lane + 32 * v) * 8);
        uh[v] = e;
        const uint4 c = make_uint4(bf2_min(bf2_max(e.x, 0xc61cc61cu), 0x461c461cu), bf2_min(bf2_max(e.y, 0xc61cc61cu), 0x461c461cu),
                                   bf2_min(bf2_max(e.z, 0xc61cc61cu), 0x461c461cu), bf2_min(bf2_max(e.w, 0xc61cc61cu), 0x461c461cu));
        *reinterpret_cast<uint4*>(reinterpret_cast<T*>(p.hx) + off) = one;
        *reinterpret_cast<uint4*>(reinterpret_cast<T*>(p.cx) + off) = e;
        *reinterpret_cast<uint4*>(reinterpret_cast<T*>(p.cxc) + off) = c;
        *reinterpret_cast<uint4*>(reinterpret_cast<T*>(p.h) + off) = e;
      }
    }
  } else {
  uint4 ua[NV], up[NV];
#pragma unroll
  for (int v = 0; v < NV; ++v) {
    const size_t off = row + (size_t)(lane + 32 * v) * 8;
    const bool act = lane + 32 * v < nch;
    ua[v] = act ? *reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(p.out0) + off) : z;
    uh[v] = act ? *reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(p.h) + off) : z;
    up[v] = act ? *reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(p.hx_pre) + off) : z;
  }
  // out = norm(out0 + down_proj(...)) (:571-573), h += out (:793), hx = norm(hx + hx_moe) (:563-564)
  float ss0 = 0.f, ss1 = 0.f;
#pragma unroll
  for (int v = 0; v < NV; ++v)
    if (lane + 32 * v < nch) {
      float a[8], hp[8];
      unpack8(ua[v], a);
      unpack8(up[v], hp);
      ss0 += sumsq8(a);
      ss1 += sumsq8(hp);
    }
  ss0 = warp_sum(ss0);
  ss1 = warp_sum(ss1);
#pragma unroll
  for (int v = 0; v < NV; ++v)
    if (lane + 32 * v < nch) {
      const int c = lane + 32 * v;
      const size_t off = row + (size_t)c * 8;
      float pw[8], pb[8], x[8], b[8], h[8];
      load8(reinterpret_cast<const T*>(p.prev_norm_w) + c * 8, pw);
      if (p.prev_norm_b) load8(reinterpret_cast<const T*>(p.prev_norm_b) + c * 8, pb);
      unpack8(ua[v], x);
      chunk_norm_r<T>(x, ss0, D, 1e-6f, pw, pb, p.prev_norm_b != nullptr, b);
      unpack8(uh[v], h);
#pragma unroll
      for (int e = 0; e < 8; ++e) h[e] = rnd<T>(h[e] + b[e]);
      unpack8(up[v], x);
      chunk_norm_r<T>(x, ss1, D, 1e-6f, pw, pb, p.prev_norm_b != nullptr, b);
      store8(reinterpret_cast<T*>(p.hx) + off, b);
      store8(reinterpret_cast<T*>(p.h) + off, h);
      uh[v] = make_uint4(pack_bf16x2(h[0], h[1]), pack_bf16x2(h[2], h[3]), pack_bf16x2(h[4], h[5]),
                         pack_bf16x2(h[6], h[7]));
    }
  }
  // PRE_FINAL: the lm-head-side norm of h; otherwise norm_x = norm1(h) (:340)
  float s3 = 0.f;
#pragma unroll
  for (int v = 0; v < NV; ++v)
    if (lane + 32 * v < nch) {
      float h[8];
      unpack8(uh[v], h);
      s3 += sumsq8(h);
    }
  s3 = warp_sum(s3);
#pragma unroll
  for (int v = 0; v < NV; ++v)
    if (lane + 32 * v < nch) {
      const int c = lane + 32 * v;
      float w1[8], h[8], b[8];
      unpack8(uh[v], h);
      if (p.mode == PRE_FINAL) {
        chunk_norm<T>(h, s3, D, p.lhs_eps, reinterpret_cast<const T*>(p.lhs_w), reinterpret_cast<const T*>(p.lhs_b), c, b);
        store8(reinterpret_cast<T*>(p.hf) + row + (size_t)c * 8, b);
        continue;
      }
      load8(reinterpret_cast<const T*>(p.norm1_w) + c * 8, w1);
      chunk_norm_r<T>(h, s3, D, 1e-6f, w1, w1, false, b);
      store8(reinterpret_cast<T*>(p.norm_x) + row + (size_t)c * 8, b);
    }
}

// ------------------------------------------------------------------ prefill prefix mean
// cumsum over the sequence in fp32 (CPU cumsum accumulates in order, in fp32) divided
// by the arange divisors (:376-387). One thread per (sequence, feature).
struct ScanParams {
  int B, S, D;
  const void* norm_x;   // [B, S, D]
  void* mean;           // [B, S, D]
  float* state;         // [B, D] running sum in / out (decode state after the prompt)
  const float* div;     // [S] divisor of each prompt position
  const float2* dr;     // [S] (div, RN(1 / div)) of each prompt position (bf16 models), or null
};

// a / b rounded to nearest-even in fp32, given y = RN(1 / b), by one residual correction
// (Markstein, "Computation of elementary functions on the IBM RISC System/6000 processor",
// IBM J. Res. Dev. 34(1), 1990: with y the correctly rounded reciprocal and q0 a faithful
// quotient, q0 + (a - b q0) y rounded once is the correctly rounded quotient; the residual
// is exact under FMA). An exact q0 and a non-finite q0 are returned as they are. The engine
// uses it for bf16 dividends and the prompt divisors; a GPU test checks it against the
// division for every bf16 dividend and every divisor of positions 1..16384.
ONE_DEVINL float div_rn_recip(float a, float b, float y) {
  const float q0 = a * y;
  const float r = fmaf(-q0, b, a);
  return (r == 0.f || !(fabsf(q0) <= 3.402823466e38f)) ? q0 : fmaf(r, y, q0);
}

// two consecutive elements <-> two floats
ONE_DEVINL void ld2(const __nv_bfloat16* p, float& a, float& b) {
  const uint32_t u = *reinterpret_cast<const uint32_t*>(p);
  a = __uint_as_float(u << 16);
  b = __uint_as_float(u & 0xffff0000u);
}
ONE_DEVINL void ld2(const float* p, float& a, float& b) {
  const float2 v = *reinterpret_cast<const float2*>(p);
  a = v.x;
  b = v.y;
}
ONE_DEVINL void st2(__nv_bfloat16* p, float a, float b) { *reinterpret_cast<uint32_t*>(p) = pack_bf16x2(a, b); }
ONE_DEVINL void st2(float* p, float a, float b) { *reinterpret_cast<float2*>(p) = make_float2(a, b); }

template <typename T>
__global__ void __launch_bounds__(256) scan_mean_kernel(const ScanParams p) {
  pdl_launch_dependents();
  pdl_wait();
  // one thread per (sequence, feature pair): the prefix sum runs in token order in fp32 (the
  // reference's CPU cumsum order). The next 32 tokens' input pairs and divisors are loaded
  // before the adds; every mean pair is one store.
  constexpr int kAhead = 32;
  const int half = p.D / 2;
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= p.B * half) return;
  const int bb = idx / half, d = 2 * (idx % half);
  float a0 = p.state[(size_t)bb * p.D + d], a1 = p.state[(size_t)bb * p.D + d + 1];
  const T* __restrict__ x = reinterpret_cast<const T*>(p.norm_x) + (size_t)bb * p.S * p.D + d;
  T* __restrict__ m = reinterpret_cast<T*>(p.mean) + (size_t)bb * p.S * p.D + d;
  const float* __restrict__ div = p.div;
  if constexpr (sizeof(T) == 2) {
    if (p.dr) {
      // bf16 with the (divisor, reciprocal) table: input pairs as packed words; the next 32
      // tokens' loads are in flight while the current 32 are summed and divided
      constexpr int kA = 32;
      const uint32_t* __restrict__ x32 = reinterpret_cast<const uint32_t*>(x);
      uint32_t* __restrict__ m32 = reinterpret_cast<uint32_t*>(m);
      const float2* __restrict__ dr = p.dr;
      const size_t rs = (size_t)(p.D / 2);
      uint32_t vc[kA], vn[kA];
#pragma unroll
      for (int j = 0; j < kA; ++j)
        if (j < p.S) vc[j] = x32[(size_t)j * rs];
      for (int s0 = 0; s0 < p.S; s0 += kA) {
        const int n = min(kA, p.S - s0), nn = min(kA, p.S - s0 - kA);
#pragma unroll
        for (int j = 0; j < kA; ++j)
          if (j < nn) vn[j] = x32[(size_t)(s0 + kA + j) * rs];
#pragma unroll
        for (int j = 0; j < kA; ++j)
          if (j < n) {
            a0 += bf2_lo(vc[j]);
            a1 += bf2_hi(vc[j]);
            const float2 q = __ldg(dr + s0 + j);
            m32[(size_t)(s0 + j) * rs] = pack_bf16x2(div_rn_recip(rnd<T>(a0), q.x, q.y), div_rn_recip(rnd<T>(a1), q.x, q.y));
          }
#pragma unroll
        for (int j = 0; j < kA; ++j) vc[j] = vn[j];
      }
      p.state[(size_t)bb * p.D + d] = a0;
      p.state[(size_t)bb * p.D + d + 1] = a1;
      return;
    }
  }
  for (int s0 = 0; s0 < p.S; s0 += kAhead) {
    const int n = min(kAhead, p.S - s0);
    float v0[kAhead], v1[kAhead], dv[kAhead];
#pragma unroll
    for (int j = 0; j < kAhead; ++j)
      if (j < n) {
        ld2(x + (size_t)(s0 + j) * p.D, v0[j], v1[j]);
        dv[j] = __ldg(div + s0 + j);
      }
#pragma unroll
    for (int j = 0; j < kAhead; ++j)
      if (j < n) {
        a0 += v0[j];
        a1 += v1[j];
        st2(m + (size_t)(s0 + j) * p.D, rnd<T>(a0) / dv[j], rnd<T>(a1) / dv[j]);
      }
  }
  p.state[(size_t)bb * p.D + d] = a0;
  p.state[(size_t)bb * p.D + d + 1] = a1;
}

// Prefix mean of bf16 prompts with the (divisor, reciprocal) table, staged through shared
// memory: a CTA owns one sequence and 64 features (64 threads, one feature each: the sums
// are sequential in the token, so B x D chains are all the parallelism there is) and keeps
// kScanStages - 1 tiles of kScanTok tokens x 128 bytes in flight with cp.async, so the fp32
// sums read from shared memory while HBM streams the next tiles. Same arithmetic, in the
// same order, as scan_mean_kernel's bf16 path.
constexpr int kScanTok = 64;
constexpr int kScanStages = 4;
constexpr int kScanThreads = 64;
constexpr int kScanFeat = kScanThreads;
constexpr size_t kScanSmem = (size_t)kScanStages * kScanTok * (kScanFeat * 2 + 8);

__global__ void __launch_bounds__(kScanThreads) scan_mean_staged_kernel(const ScanParams p) {
  using T = __nv_bfloat16;
  extern __shared__ __align__(16) uint32_t ssm[];
  pdl_launch_dependents();
  const int groups = p.D / kScanFeat;
  const int bb = blockIdx.x / groups, g = blockIdx.x % groups, tid = threadIdx.x;
  const int d = g * kScanFeat + tid;
  uint16_t* xs = reinterpret_cast<uint16_t*>(ssm);  // [stage][token][feature]
  float2* ds = reinterpret_cast<float2*>(ssm + (size_t)kScanStages * kScanTok * kScanFeat / 2);  // [stage][token]
  const size_t row = (size_t)p.D * 2;
  const uint8_t* xg = reinterpret_cast<const uint8_t*>(p.norm_x) + ((size_t)bb * p.S * p.D + g * kScanFeat) * 2;
  uint16_t* mg = reinterpret_cast<uint16_t*>(p.mean) + (size_t)bb * p.S * p.D + d;
  const int nst = (p.S + kScanTok - 1) / kScanTok;
  constexpr int kChunks = kScanFeat * 2 / 16;  // 16-byte chunks of a token's slice
  pdl_wait();
  float a0 = p.state[(size_t)bb * p.D + d];
  // tile st: kScanTok rows of kChunks chunks, and its kScanTok table entries; an empty group
  // past the end keeps the group count uniform
  auto issue = [&](int st) {
    if (st < nst) {
      const int s0 = st * kScanTok, n = min(kScanTok, p.S - s0);
      uint16_t* dst = xs + (size_t)(st % kScanStages) * kScanTok * kScanFeat;
      for (int c = tid; c < n * kChunks; c += kScanThreads) {
        const int t = c / kChunks, q = c % kChunks;
        cp_async16(dst + t * kScanFeat + q * 8, xg + (size_t)(s0 + t) * row + q * 16);
      }
      if (tid < n) cp_async8(ds + (st % kScanStages) * kScanTok + tid, p.dr + s0 + tid);
    }
    cp_async_commit();
  };
#pragma unroll
  for (int st = 0; st < kScanStages - 1; ++st) issue(st);
  for (int st = 0; st < nst; ++st) {
    issue(st + kScanStages - 1);
    cp_async_wait<kScanStages - 1>();  // tile st has landed (this thread's copies)
    __syncthreads();                   // ... and every other thread's
    const uint16_t* xv = xs + (size_t)(st % kScanStages) * kScanTok * kScanFeat + tid;
    const float2* dv = ds + (st % kScanStages) * kScanTok;
    const int s0 = st * kScanTok, n = min(kScanTok, p.S - s0);
    uint16_t* mo = mg + (size_t)s0 * p.D;
    if (n == kScanTok) {
#pragma unroll 16
      for (int j = 0; j < kScanTok; ++j) {
        const float2 q = dv[j];
        a0 += __uint_as_float((uint32_t)xv[j * kScanFeat] << 16);
        mo[(size_t)j * p.D] = (uint16_t)(pack_bf16x2(div_rn_recip(rnd<T>(a0), q.x, q.y), 0.f) & 0xffffu);
      }
    } else {
      for (int j = 0; j < n; ++j) {
        const float2 q = dv[j];
        a0 += __uint_as_float((uint32_t)xv[j * kScanFeat] << 16);
        mo[(size_t)j * p.D] = (uint16_t)(pack_bf16x2(div_rn_recip(rnd<T>(a0), q.x, q.y), 0.f) & 0xffffu);
      }
    }
    __syncthreads();  // the tile's buffer is refilled by the next iteration's issue
  }
  cp_async_wait<0>();
  p.state[(size_t)bb * p.D + d] = a0;
}

// ------------------------------------------------------------------ final norm
struct RowNormParams {
  int T, D;
  const void* in;
  void* out;
  const void* w;
  const void* b;
  float eps;
  int* counters;      // non-null: advance {pos, step} (end of a decode step)
  int in_row_mul;     // input row of output row t: t * in_row_mul + in_row_add
  int in_row_add;
};

template <typename T, int NV>
__global__ void __launch_bounds__(256) row_norm_kernel(const RowNormParams p) {
  pdl_launch_dependents();
  pdl_wait();
  if (p.counters && blockIdx.x == 0 && threadIdx.x == 0) {
    p.counters[0] += 1;
    p.counters[1] += 1;
  }
  const int warps = blockDim.x >> 5;
  const int t = blockIdx.x * warps + (threadIdx.x >> 5);
  if (t >= p.T) return;
  const int nch = p.D / 8;
  float x[NV][8], y[NV][8];
  warp_load_row<T, NV>(reinterpret_cast<const T*>(p.in) + ((size_t)t * p.in_row_mul + p.in_row_add) * p.D, nch, x);
  warp_rmsnorm<T, NV>(x, nch, reinterpret_cast<const T*>(p.w), reinterpret_cast<const T*>(p.b), p.eps, p.D, y);
  warp_store_row<T, NV>(reinterpret_cast<T*>(p.out) + (size_t)t * p.D, nch, y);
}

// ------------------------------------------------------------------ attention + routers
struct MoeRouter {
  const void* gate_w;   // [r, in] (null: gate logits precomputed in glog)
  const void* glog;     // [T, r] precomputed gate logits (cx_moe)
  const void* experts;  // [E]
  const void* bias2;    // [E, in]
  const void* x;        // [T, ldx] router input (already clamped for cx)
  int ldx;
  int in;
  void* comb;           // [T, in] combined input of the shared Linear
  int* idx_out;         // [T, k] chosen experts (optional)
};

struct RowAttnParams {
  int T, H, Dh, r, E, k, use_moe;
  int seq_len;            // prefill: position = pos0 + t % seq_len; decode: seq_len = 0
  const int* counters;    // {pos, step}
  const float* inv_freq;  // [Dh/2]
  const void* proj;       // [T, 3*H*Dh]: lin1 | lin2 | lin3 outputs (bias added)
  float attn_scale;
  const void* wq; const void* bq;  // lin_q [H, Dh], [H]
  const void* wk; const void* bk;
  const void* wv; const void* bv;
  void* o;                // [T, H*H] attention output (plain-Linear path input), optional
  MoeRouter rt[3];        // hx_moe, x_moe, cx_moe
  unsigned long long tie; // topk_tie_selection(E, k)
  DevErr* err;
};

// Shared-memory layout of row_attn_kernel (byte offsets), shared by host and device.
constexpr int kAttnTok = 2;            // tokens per CTA iteration
constexpr int kAttnThreads = 384;      // 12 warps: per token 1 (hx_moe) + 1 (x_moe) + 4 (cx_moe)
constexpr int kAttnCxWarps = 4;
struct AttnTokLayout {
  int row, cs, rot, qkv, o, xs, cxs, gl, gq, cv, part, scr, sc, sel, bytes;
};
struct AttnLayout {
  int wqkv, bqkv, gate, gate_ld, experts, b2, tok0, total;
  int wq16, g16;  // staged bf16 copies of lin_q/k/v [3][H][Dh] and the hx/x gates [2][r][HH] (0 bytes if not staged)
  bool staged;
  AttnTokLayout tk;
};
__host__ __device__ inline int attn_take(int& off, int bytes) {
  const int o = off;
  off = (off + bytes + 15) & ~15;
  return o;
}
// stage_w: copy the tensor-core operands read by every token (lin_q/k/v, the hx/x gate
// weights) into shared memory before the dependency wait (decode); prompt ingestion runs two
// CTAs per SM and reads them through L1 instead.
__host__ __device__ inline AttnLayout attn_layout(int H, int Dh, int r, int E, int D, int use_moe, int es,
                                                  int stage_w = 0) {
  AttnLayout L;
  int off = 0;
  const int HD = H * Dh, HH = H * H, Dp = Dh + 4;
  L.staged = stage_w && es == 2 && H <= 16;
  L.wq16 = attn_take(off, L.staged ? 3 * HD * 2 : 0);
  L.g16 = attn_take(off, L.staged && use_moe && HH % 16 == 0 ? 2 * r * HH * 2 : 0);
  L.wqkv = attn_take(off, (es == 4 || H > 16) ? 3 * H * Dp * 4 : 0);  // CUDA-core projections only
  L.bqkv = attn_take(off, 3 * H * 4);
  L.gate_ld = HH + (es == 2 ? 2 : 1);  // odd row stride in 32-bit words: conflict-free rows
  L.gate = attn_take(off, 0);  // the router weights are read where they are used (L1/L2)
  L.experts = attn_take(off, use_moe ? 3 * E * 4 : 0);
  L.b2 = attn_take(off, use_moe ? E * (2 * HH + D) * es : 0);
  L.tok0 = off;
  int t = 0;
  AttnTokLayout& k = L.tk;
  k.row = attn_take(t, 3 * HD * 4);
  k.cs = attn_take(t, 2 * Dh * 4);
  k.rot = attn_take(t, H * 2 * Dp * 4);
  k.qkv = attn_take(t, H * 3 * H * 4);
  k.o = attn_take(t, HH * 4);
  k.xs = attn_take(t, HH * 4);
  k.cxs = attn_take(t, use_moe ? D * 4 : 0);
  k.gl = attn_take(t, 3 * r * 4);
  k.gq = attn_take(t, kAttnCxWarps * r * 4);          // per cx warp copy of the gate logits
  k.cv = attn_take(t, (2 + kAttnCxWarps) * E * 4);
  k.part = attn_take(t, kAttnCxWarps * kMaxExperts * 8);  // cx expert partial sums
  k.scr = attn_take(t, 6 * 32 * 8);                   // per router warp scratch
  k.sc = attn_take(t, 3 * E * 4);
  k.sel = attn_take(t, 3 * E * 4);
  k.bytes = t;
  L.total = off + kAttnTok * t;
  return L;
}

// D += A * B for one m16n8k16 tile, bf16 inputs, fp32 accumulators (warp-wide).
ONE_DEVINL void mma_16816_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
ONE_DEVINL uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}
ONE_DEVINL uint32_t ldg_u32(const void* p) { return *reinterpret_cast<const uint32_t*>(p); }

ONE_DEVINL void named_bar(int id, int nthreads) { named_barrier_sync(id, nthreads); }

// softmax over the r gate logits in g[] (fp32, cast to the dtype), then the expert
// factors c_e = 1 + silu(clamp(mean_r(rnd(g * e)))) (one/linear_moe.py:56-68) into c[].
// One warp; `cp` is 32 doubles of scratch.
template <typename T>
ONE_DEVINL void warp_gate_factors_loop(float* g, int r, const float* ex, int E, float* c, double* cp) {
  const int lane = threadIdx.x & 31;
  float mx = -INFINITY;
  for (int j = lane; j < r; j += 32) mx = fmaxf(mx, g[j]);
  mx = warp_max(mx);
  float sum = 0.f;
  for (int j = lane; j < r; j += 32) sum += expf(g[j] - mx);
  sum = warp_sum(sum);
  const float inv = 1.0f / sum;
  __syncwarp();
  for (int j = lane; j < r; j += 32) g[j] = rnd<T>(expf(g[j] - mx) * inv);
  __syncwarp();
  for (int e0 = 0; e0 < E; e0 += 32) {
    const int ne = min(32, E - e0);
    const int slices = 32 / ne;
    const int e = lane % ne, sl = lane / ne;
    double acc = 0.0;
    if (sl < slices)
      for (int j = sl; j < r; j += slices) acc += (double)rnd<T>(g[j] * ex[e0 + e]);
    cp[lane] = acc;
    __syncwarp();
    if (lane < ne) {
      double s2 = 0.0;
      for (int q = 0; q < slices; ++q) s2 += cp[q * ne + lane];
      const float scv = fminf(fmaxf(rnd<T>((float)s2 / (float)r), -10.f), 10.f);
      c[e0 + lane] = rnd<T>(1.0f + rnd<T>(silu_f(scv)));
    }
    __syncwarp();
  }
}

// Gate softmax (one/linear_moe.py:56) and expert factors c_e = 1 + silu(clamp(mean_j
// rnd(gate_j * experts_e))) (:59-68) for one token, one warp. r <= 128: each lane keeps its gate
// entries in registers, computes each exponential once, and accumulates the products for all
// experts; the per-expert sums are exact (fp64 sums of bf16 terms), so the order of the
// warp reduction does not change them. Larger r takes warp_gate_factors_loop.
template <typename T>
ONE_DEVINL void warp_gate_factors(float* g, int r, const float* ex, int E, float* c, double* cp) {
  constexpr int kPer = 4;
  if (r > 32 * kPer) {
    warp_gate_factors_loop<T>(g, r, ex, E, c, cp);
    return;
  }
  const int lane = threadIdx.x & 31;
  float gv[kPer];
  float mx = -INFINITY;
#pragma unroll
  for (int m = 0; m < kPer; ++m) {
    const int j = lane + 32 * m;
    gv[m] = j < r ? g[j] : -INFINITY;
    mx = fmaxf(mx, gv[m]);
  }
  mx = warp_max(mx);
  float sum = 0.f;
#pragma unroll
  for (int m = 0; m < kPer; ++m) {
    gv[m] = lane + 32 * m < r ? expf(gv[m] - mx) : 0.f;
    sum += gv[m];
  }
  sum = warp_sum(sum);
  const float inv = 1.0f / sum;
  if constexpr (sizeof(T) == 2) {
    // rounded gate values as bf16x2 pairs (m = 0, 1) and (2, 3); products rnd(g * x_e) are
    // one packed multiply each; per-expert totals by the transposed butterfly
    const uint32_t gp0 = pack_bf16x2(gv[0] * inv, gv[1] * inv), gp1 = pack_bf16x2(gv[2] * inv, gv[3] * inv);
    const bool two = r > 64;
    const int slot = r2_slot(lane);
    for (int e0 = 0; e0 < E; e0 += 8) {
      double a[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const uint32_t xe2 = e0 + e < E ? bf2_splat(ex[e0 + e]) : 0u;
        const uint32_t p0 = bf2_mul(gp0, xe2);
        a[e] = (double)bf2_lo(p0);
        a[e] += (double)bf2_hi(p0);
        if (two) {
          const uint32_t p1 = bf2_mul(gp1, xe2);
          a[e] += (double)bf2_lo(p1);
          a[e] += (double)bf2_hi(p1);
        }
      }
      const double tot = warp_transpose_sum8(a);
      if ((lane & 3) == 0 && e0 + slot < E) {
        const float scv = fminf(fmaxf(rnd<T>((float)tot / (float)r), -10.f), 10.f);
        c[e0 + slot] = rnd<T>(1.0f + rnd<T>(silu_f(scv)));
      }
    }
    __syncwarp();
  } else {
#pragma unroll
    for (int m = 0; m < kPer; ++m) gv[m] = rnd<T>(gv[m] * inv);
    for (int e0 = 0; e0 < E; e0 += 8) {
      double acc[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        acc[e] = 0.0;
        if (e0 + e < E) {
          const float xe = ex[e0 + e];
#pragma unroll
          for (int m = 0; m < kPer; ++m)
            if (lane + 32 * m < r) acc[e] += (double)rnd<T>(gv[m] * xe);
        }
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] = warp_sum_d(acc[e]);
      double mine = acc[0];
#pragma unroll
      for (int e = 1; e < 8; ++e)
        if (lane == e) mine = acc[e];
      if (lane < 8 && e0 + lane < E) {
        const float scv = fminf(fmaxf(rnd<T>((float)mine / (float)r), -10.f), 10.f);
        c[e0 + lane] = rnd<T>(1.0f + rnd<T>(silu_f(scv)));
      }
    }
    __syncwarp();
  }
}

// Per-expert sums over x[i0..i1) of rnd(rnd(x * c_e) + bias2[e, i]) for experts e0..e0+7,
// reduced over the warp (exact fp64); returns the total of expert e0 + r2_slot(lane). bf16
// with even bounds and 4-byte aligned rows: each lane takes input pairs, rounds x * c_e and
// the biased sum as packed bf16x2 operations (the inputs are bf16 values) and adds both
// halves in fp64. The terms are bf16 numbers, so their fp64 sum does not depend on the order.
template <typename T>
ONE_DEVINL double warp_expert_sums_t(const float* x, int i0, int i1, const T* B2, int in, const float* c, int e0, int E) {
  const int lane = threadIdx.x & 31;
  double acc[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) acc[e] = 0.0;
  const int ne = min(8, E - e0);
  if (sizeof(T) == 2 && ((i0 | i1 | in) & 1) == 0 && (reinterpret_cast<uintptr_t>(B2) & 3) == 0 &&
      (reinterpret_cast<uintptr_t>(x) & 7) == 0) {
    uint32_t c2[8];
    const uint32_t* brow[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      c2[e] = e < ne ? bf2_splat(c[e0 + e]) : 0u;
      brow[e] = reinterpret_cast<const uint32_t*>(B2 + (size_t)(e0 + (e < ne ? e : 0)) * in);
    }
    for (int i = i0 + 2 * lane; i < i1; i += 64) {
      const float2 xv = *reinterpret_cast<const float2*>(x + i);
      const uint32_t xp = pack_bf16x2(xv.x, xv.y);
#pragma unroll
      for (int e = 0; e < 8; ++e)
        if (e < ne) {
          const uint32_t r = bf2_add(bf2_mul(xp, c2[e]), brow[e][i >> 1]);
          acc[e] += (double)bf2_lo(r);
          acc[e] += (double)bf2_hi(r);
        }
    }
  } else {
    for (int i = i0 + lane; i < i1; i += 32) {
      const float xi = x[i];
#pragma unroll
      for (int e = 0; e < 8; ++e)
        if (e0 + e < E) {
          const float cv = c[e0 + e];
          const float xc = cv == 1.0f ? xi : rnd<T>(xi * cv);
          acc[e] += (double)rnd<T>(xc + ld<T>(B2 + (size_t)(e0 + e) * in + i));
        }
    }
  }
  return warp_transpose_sum8(acc);
}

// mean of the selected biased inputs over x[i0..i1) (one/linear_moe.py:87-90): fp32 sum in
// selection order, divided by k, rounded once
template <typename T>
ONE_DEVINL void warp_combine(const float* x, int i0, int i1, const T* B2, int in, const float* c, const int* sel, int kk,
                             T* out) {
  const int lane = threadIdx.x & 31;
  if (sizeof(T) == 2 && kk <= 8 && ((i0 | i1 | in) & 1) == 0 && (reinterpret_cast<uintptr_t>(B2) & 3) == 0 &&
      (reinterpret_cast<uintptr_t>(x) & 7) == 0 && (reinterpret_cast<uintptr_t>(out) & 3) == 0) {
    // packed: rnd(x * c_e) and the biased sum as bf16x2 operations, fp32 sums in selection order
    uint32_t c2[8];
    const uint32_t* brow[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int e = j < kk ? sel[j] : 0;
      c2[j] = bf2_splat(c[e]);
      brow[j] = reinterpret_cast<const uint32_t*>(B2 + (size_t)e * in);
    }
    const bool pow2 = (kk & (kk - 1)) == 0;
    const float invk = 1.0f / (float)kk;
    for (int i = i0 + 2 * lane; i < i1; i += 64) {
      const float2 xv = *reinterpret_cast<const float2*>(x + i);
      const uint32_t xp = pack_bf16x2(xv.x, xv.y);
      float s0 = 0.f, s1 = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (j < kk) {
          const uint32_t r = bf2_add(bf2_mul(xp, c2[j]), brow[j][i >> 1]);
          s0 += bf2_lo(r);
          s1 += bf2_hi(r);
        }
      *reinterpret_cast<uint32_t*>(out + i) =
          pow2 ? pack_bf16x2(s0 * invk, s1 * invk) : pack_bf16x2(s0 / (float)kk, s1 / (float)kk);
    }
    return;
  }
  for (int i = i0 + lane; i < i1; i += 32) {
    float s2 = 0.f;
    for (int j = 0; j < kk; ++j) {
      const int e = sel[j];
      s2 += rnd<T>(rnd<T>(x[i] * c[e]) + ld<T>(B2 + (size_t)e * in + i));
    }
    st<T>(out + i, s2 / (float)kk);
  }
}

// Feature attention (one/modeling_one.py:390-556) and the three LinearMoE routers,
// kAttnTok tokens per CTA iteration. Every weight the kernel reads (lin_q/k/v, the
// hx_moe / x_moe gates, experts, bias2) is copied to shared memory before the
// dependency wait.
//   phase A: warp per (token, head): RoPE (rotate_half) on single_x * scale and on key,
//            lane u computes projection output u of q|k|v (Dh -> H, bias, rounded),
//            softmax(q*k - max) in fp32 over lanes j < H, o = w * v.
//   phase B: per token, warp 0 routes hx_moe, warp 1 x_moe (gate GEMV, softmax, expert
//            factors, expert sums, top-k, combine) and warps 2..5 route cx_moe, each
//            summing and combining a quarter of the 768 inputs; no CTA-wide barrier.
// MINB = 2 (prompt ingestion): two CTAs per SM, registers capped to fit both; decode keeps
// MINB = 1 for the shortest per-token chain.
template <typename T, int HMAX, int MINB = 1>
__global__ void __launch_bounds__(kAttnThreads, MINB) row_attn_kernel(const RowAttnParams p) {
  extern __shared__ __align__(16) uint8_t smb[];
  const int H = p.H, Dh = p.Dh, HD = H * Dh, HH = H * H, r = p.r, E = p.E;
  const int D = p.use_moe ? p.rt[2].in : 0;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nthr = blockDim.x, nw = nthr >> 5;
  const AttnLayout L = attn_layout(H, Dh, r, E, D, p.use_moe, (int)sizeof(T), MINB == 1 ? 1 : 0);
  float* wqkv = reinterpret_cast<float*>(smb + L.wqkv);
  float* bqkv = reinterpret_cast<float*>(smb + L.bqkv);
  float* exps = reinterpret_cast<float*>(smb + L.experts);
  const int half = Dh / 2, Dp = Dh + 4;
  const int inr[3] = {HH, HH, D};

  // ---- small weights to shared memory (not written by the previous kernel: before the wait)
  if (L.staged) {
    const uint4* src[3] = {reinterpret_cast<const uint4*>(p.wq), reinterpret_cast<const uint4*>(p.wk),
                           reinterpret_cast<const uint4*>(p.wv)};
    uint4* dst = reinterpret_cast<uint4*>(smb + L.wq16);
    const int nv = HD * 2 / 16;  // 16-byte vectors per projection
    for (int v = tid; v < 3 * nv; v += nthr) dst[v] = src[v / nv][v % nv];
    if (p.use_moe && HH % 16 == 0) {
      const int ng = r * HH * 2 / 16;
      uint4* gd = reinterpret_cast<uint4*>(smb + L.g16);
      for (int v = tid; v < 2 * ng; v += nthr)
        gd[v] = reinterpret_cast<const uint4*>(p.rt[v / ng].gate_w)[v % ng];
    }
  }
  constexpr bool kTensor = sizeof(T) == 2;  // bf16: projections and gates on mma.sync
  if constexpr (!(kTensor && HMAX <= 16))
    for (int v = tid; v < 3 * HD / 8; v += nthr) {
      const int u = (v * 8) / Dh, d0 = (v * 8) % Dh, which = u / H;
      const T* W = reinterpret_cast<const T*>(which == 0 ? p.wq : which == 1 ? p.wk : p.wv);
      float x[8];
      load8(W + (size_t)(u % H) * Dh + d0, x);
#pragma unroll
      for (int e = 0; e < 8; ++e) wqkv[u * Dp + d0 + e] = x[e];
    }
  for (int i = tid; i < 3 * H; i += nthr) {
    const int which = i / H, j = i % H;
    const T* Bb = reinterpret_cast<const T*>(which == 0 ? p.bq : which == 1 ? p.bk : p.bv);
    bqkv[i] = ld<T>(Bb + j);
  }
  T* b2s = reinterpret_cast<T*>(smb + L.b2);
  const int b2off[3] = {0, E * HH, 2 * E * HH};
  if (p.use_moe) {
    for (int i = tid; i < 3 * E; i += nthr)
      exps[i] = fminf(fmaxf(ld<T>(reinterpret_cast<const T*>(p.rt[i / E].experts) + i % E), -10.f), 10.f);
    constexpr int VE = 16 / (int)sizeof(T);
    for (int ri = 0; ri < 3; ++ri) {
      const uint4* src = reinterpret_cast<const uint4*>(p.rt[ri].bias2);
      uint4* dst = reinterpret_cast<uint4*>(b2s + b2off[ri]);
      for (int v = tid; v < E * inr[ri] / VE; v += nthr) dst[v] = src[v];
    }
  }
  if (tid == 0) pdl_launch_dependents();
  pdl_wait();

  for (int t0 = blockIdx.x * kAttnTok; t0 < p.T; t0 += gridDim.x * kAttnTok) {
    const int ntok = min(kAttnTok, p.T - t0);
    // ---- phase 0: rows of each token. The 16-byte chunks of every token's projections (and
    // cx) are loaded in batches of three per thread before any is stored, so the tokens'
    // loads are in flight together.
    {
      const int nproj = 3 * HD / 8, ncx = p.use_moe ? D / 8 : 0, per_tok = nproj + ncx;
      const int items = ntok * per_tok;
      constexpr int kBatch = 3;
      for (int base = 0; base < items; base += kBatch * nthr) {
        float v[kBatch][8];
#pragma unroll
        for (int m = 0; m < kBatch; ++m) {
          const int it = base + tid + m * nthr;
          if (it < items) {
            const int k = it / per_tok, j = it % per_tok, t = t0 + k;
            const T* src = j < nproj ? reinterpret_cast<const T*>(p.proj) + (size_t)t * 3 * HD + j * 8
                                     : reinterpret_cast<const T*>(p.rt[2].x) + (size_t)t * p.rt[2].ldx + (j - nproj) * 8;
            load8(src, v[m]);
          }
        }
#pragma unroll
        for (int m = 0; m < kBatch; ++m) {
          const int it = base + tid + m * nthr;
          if (it < items) {
            const int k = it / per_tok, j = it % per_tok;
            uint8_t* tb = smb + L.tok0 + k * L.tk.bytes;
            float* dst;
            if (j < nproj) {
              if (j * 8 < HD)
#pragma unroll
                for (int e = 0; e < 8; ++e) v[m][e] = rnd<T>(v[m][e] * p.attn_scale);  // :405
              dst = reinterpret_cast<float*>(tb + L.tk.row) + j * 8;
            } else {
              dst = reinterpret_cast<float*>(tb + L.tk.cxs) + (j - nproj) * 8;
            }
#pragma unroll
            for (int e = 0; e < 8; ++e) dst[e] = v[m][e];
          }
        }
      }
      // cos / sin (OneRotaryEmbedding, :159-182): fp32 inv_freq * pos, cast to the dtype
      for (int it = tid; it < ntok * half; it += nthr) {
        const int k = it / half, i = it % half, t = t0 + k;
        float* cs = reinterpret_cast<float*>(smb + L.tok0 + k * L.tk.bytes + L.tk.cs);
        const int pos = p.counters[0] + (p.seq_len > 0 ? t % p.seq_len : 0);
        const float f = p.inv_freq[i] * (float)pos;
        const float c = rnd<T>(cosf(f)), sn = rnd<T>(sinf(f));
        cs[i] = c; cs[i + half] = c;
        cs[Dh + i] = sn; cs[Dh + i + half] = sn;
      }
      if (p.use_moe)
        for (int it = tid; it < ntok * r; it += nthr) {
          const int k = it / r, j = it % r;
          float* gl = reinterpret_cast<float*>(smb + L.tok0 + k * L.tk.bytes + L.tk.gl);
          gl[2 * r + j] = ld<T>(reinterpret_cast<const T*>(p.rt[2].glog) + (size_t)(t0 + k) * r + j);
        }
    }
    __syncthreads();

    // ---- phase A
    // HMAX = 16 instantiations only run H <= 16: the CUDA-core path below is not compiled
    // into them (instruction-cache pressure)
    constexpr bool mmaA = kTensor && HMAX <= 16;
    if constexpr (mmaA) {
      // warp per head, both tokens at once: RoPE into shared rows, then q|k|v = x @ W^T on
      // mma.sync (the tokens are the M rows of an m16n8k16 tile), bias, rounding, softmax.
      for (int h = warp; h < H; h += nw) {
        for (int k = 0; k < ntok; ++k) {
          uint8_t* tb = smb + L.tok0 + k * L.tk.bytes;
          const float* row = reinterpret_cast<const float*>(tb + L.tk.row);
          const float* cs = reinterpret_cast<const float*>(tb + L.tk.cs);
          float* xr = reinterpret_cast<float*>(tb + L.tk.rot) + h * 2 * Dp;
          float* kr = xr + Dp;
          const float* sx = row + h * Dh;
          const float* sk = row + HD + h * Dh;
          for (int d = lane; d < Dh; d += 32) {
            const float px = d < half ? -sx[d + half] : sx[d - half];
            const float pk = d < half ? -sk[d + half] : sk[d - half];
            xr[d] = rnd<T>(rnd<T>(sx[d] * cs[d]) + rnd<T>(px * cs[Dh + d]));
            kr[d] = rnd<T>(rnd<T>(sk[d] * cs[d]) + rnd<T>(pk * cs[Dh + d]));
          }
        }
        __syncwarp();
        const int g = lane >> 2, c = lane & 3;
        const bool rowok = g < ntok;
        const float* srcs[3] = {nullptr, nullptr, nullptr};
        if (rowok) {
          uint8_t* tb = smb + L.tok0 + g * L.tk.bytes;
          float* xr = reinterpret_cast<float*>(tb + L.tk.rot) + h * 2 * Dp;
          srcs[0] = xr;
          srcs[1] = xr + Dp;
          srcs[2] = reinterpret_cast<const float*>(tb + L.tk.row) + 2 * HD + h * Dh;
        }
        const T* Ws[3] = {reinterpret_cast<const T*>(p.wq), reinterpret_cast<const T*>(p.wk), reinterpret_cast<const T*>(p.wv)};
        if (L.staged)
#pragma unroll
          for (int pj = 0; pj < 3; ++pj) Ws[pj] = reinterpret_cast<const T*>(smb + L.wq16) + pj * HD;
        float acc[3][2][4];
#pragma unroll
        for (int pj = 0; pj < 3; ++pj)
#pragma unroll
          for (int nt = 0; nt < 2; ++nt)
#pragma unroll
            for (int q = 0; q < 4; ++q) acc[pj][nt][q] = 0.f;
        for (int ks = 0; ks < Dh; ks += 16) {
#pragma unroll
          for (int pj = 0; pj < 3; ++pj) {
            uint32_t a[4] = {0u, 0u, 0u, 0u};
            if (rowok) {
              a[0] = pack_bf16(srcs[pj][ks + 2 * c], srcs[pj][ks + 2 * c + 1]);
              a[2] = pack_bf16(srcs[pj][ks + 2 * c + 8], srcs[pj][ks + 2 * c + 9]);
            }
#pragma unroll
            for (int nt = 0; nt < 2; ++nt) {
              const int n = nt * 8 + g;
              uint32_t b0 = 0u, b1 = 0u;
              if (n < H) {
                const T* wr = Ws[pj] + (size_t)n * Dh + ks + 2 * c;
                b0 = ldg_u32(wr);
                b1 = ldg_u32(wr + 8);
              }
              mma_16816_bf16(acc[pj][nt], a, b0, b1);
            }
          }
        }
        // lane (g, c) holds token g's outputs j = nt * 8 + 2c + {0, 1}
        float lg[4], vv[4];
        float mx = -INFINITY;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int nt = q >> 1, j = nt * 8 + 2 * c + (q & 1);
          lg[q] = -INFINITY;
          vv[q] = 0.f;
          if (rowok && j < H) {
            const float qv = rnd<T>(acc[0][nt][q & 1] + bqkv[j]);
            const float kv = rnd<T>(acc[1][nt][q & 1] + bqkv[H + j]);
            vv[q] = rnd<T>(acc[2][nt][q & 1] + bqkv[2 * H + j]);
            lg[q] = rnd<T>(qv * kv);
            mx = fmaxf(mx, lg[q]);
          }
        }
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        float m2 = -INFINITY;
#pragma unroll
        for (int q = 0; q < 4; ++q)
          if (lg[q] != -INFINITY) {
            lg[q] = rnd<T>(lg[q] - mx);
            m2 = fmaxf(m2, lg[q]);
          }
        m2 = fmaxf(m2, __shfl_xor_sync(0xffffffffu, m2, 1));
        m2 = fmaxf(m2, __shfl_xor_sync(0xffffffffu, m2, 2));
        float ex[4], sum = 0.f;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          ex[q] = lg[q] != -INFINITY ? expf(lg[q] - m2) : 0.f;
          sum += ex[q];
        }
        sum += __shfl_xor_sync(0xffffffffu, sum, 1);
        sum += __shfl_xor_sync(0xffffffffu, sum, 2);
        if (rowok) {
          uint8_t* tb = smb + L.tok0 + g * L.tk.bytes;
          float* o = reinterpret_cast<float*>(tb + L.tk.o);
          float* xs = reinterpret_cast<float*>(tb + L.tk.xs);
          const float inv = 1.0f / sum;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int j = (q >> 1) * 8 + 2 * c + (q & 1);
            if (j < H) {
              float w = ex[q] * inv;
              w = isnan(w) ? 1.0f / (float)H : rnd<T>(w);
              const float ov = rnd<T>(w * vv[q]);
              o[h * H + j] = ov;
              xs[h * H + j] = moe_clamp<T>(ov);  // LinearMoE clamp (:53)
            }
          }
        }
        __syncwarp();
      }
    }
    for (int pr_ = warp; !mmaA && pr_ < ntok * H; pr_ += nw) {
      const int k = pr_ / H, h = pr_ % H;
      uint8_t* tb = smb + L.tok0 + k * L.tk.bytes;
      const float* row = reinterpret_cast<const float*>(tb + L.tk.row);
      const float* cs = reinterpret_cast<const float*>(tb + L.tk.cs);
      float* xr = reinterpret_cast<float*>(tb + L.tk.rot) + h * 2 * Dp;
      float* kr = xr + Dp;
      float* qh = reinterpret_cast<float*>(tb + L.tk.qkv) + h * 3 * H;
      const float* sx = row + h * Dh;
      const float* sk = row + HD + h * Dh;
      const float* sv = row + 2 * HD + h * Dh;
      for (int d = lane; d < Dh; d += 32) {
        const float px = d < half ? -sx[d + half] : sx[d - half];
        const float pk = d < half ? -sk[d + half] : sk[d - half];
        xr[d] = rnd<T>(rnd<T>(sx[d] * cs[d]) + rnd<T>(px * cs[Dh + d]));
        kr[d] = rnd<T>(rnd<T>(sk[d] * cs[d]) + rnd<T>(pk * cs[Dh + d]));
      }
      __syncwarp();
      for (int u = lane; u < 3 * H; u += 32) {
        const int which = u / H;
        const float* src = which == 0 ? xr : which == 1 ? kr : sv;
        const float* w = wqkv + u * Dp;
        // four independent partial sums over 16-wide slices, added in slice order
        float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
        if (which < 2) {
#pragma unroll 2
          for (int d = 0; d < Dh; d += 16) {
            const float4 w0 = *reinterpret_cast<const float4*>(w + d), x0 = *reinterpret_cast<const float4*>(src + d);
            const float4 w1 = *reinterpret_cast<const float4*>(w + d + 4), x1 = *reinterpret_cast<const float4*>(src + d + 4);
            const float4 w2 = *reinterpret_cast<const float4*>(w + d + 8), x2 = *reinterpret_cast<const float4*>(src + d + 8);
            const float4 w3 = *reinterpret_cast<const float4*>(w + d + 12), x3 = *reinterpret_cast<const float4*>(src + d + 12);
            a0 = fmaf(w0.x, x0.x, a0); a0 = fmaf(w0.y, x0.y, a0); a0 = fmaf(w0.z, x0.z, a0); a0 = fmaf(w0.w, x0.w, a0);
            a1 = fmaf(w1.x, x1.x, a1); a1 = fmaf(w1.y, x1.y, a1); a1 = fmaf(w1.z, x1.z, a1); a1 = fmaf(w1.w, x1.w, a1);
            a2 = fmaf(w2.x, x2.x, a2); a2 = fmaf(w2.y, x2.y, a2); a2 = fmaf(w2.z, x2.z, a2); a2 = fmaf(w2.w, x2.w, a2);
            a3 = fmaf(w3.x, x3.x, a3); a3 = fmaf(w3.y, x3.y, a3); a3 = fmaf(w3.z, x3.z, a3); a3 = fmaf(w3.w, x3.w, a3);
          }
        } else {
#pragma unroll 4
          for (int d = 0; d < Dh; d += 4) {
            a0 = fmaf(w[d], src[d], a0);
            a1 = fmaf(w[d + 1], src[d + 1], a1);
            a2 = fmaf(w[d + 2], src[d + 2], a2);
            a3 = fmaf(w[d + 3], src[d + 3], a3);
          }
        }
        qh[u] = rnd<T>(((a0 + a1) + (a2 + a3)) + bqkv[u]);
      }
      __syncwarp();
      float lg = -INFINITY, v = 0.f;
      if (lane < H) {
        lg = rnd<T>(qh[lane] * qh[H + lane]);
        v = qh[2 * H + lane];
      }
      const float mx = warp_max(lg);
      const float d1 = lane < H ? rnd<T>(lg - mx) : -INFINITY;
      const float m2 = warp_max(d1);
      const float ex = lane < H ? expf(d1 - m2) : 0.f;
      const float sum = warp_sum(ex);
      if (lane < H) {
        float w = ex * (1.0f / sum);
        w = isnan(w) ? 1.0f / (float)H : rnd<T>(w);
        const float ov = rnd<T>(w * v);
        reinterpret_cast<float*>(tb + L.tk.o)[h * H + lane] = ov;
        reinterpret_cast<float*>(tb + L.tk.xs)[h * H + lane] = moe_clamp<T>(ov);  // LinearMoE clamp (:53)
      }
    }
    __syncthreads();
    if (p.o) {
      for (int k = 0; k < ntok; ++k) {
        const float* o = reinterpret_cast<const float*>(smb + L.tok0 + k * L.tk.bytes + L.tk.o);
        T* O = reinterpret_cast<T*>(p.o) + (size_t)(t0 + k) * HH;
        for (int i = tid; i < HH; i += nthr) st<T>(O + i, o[i]);
      }
    }
    if (p.use_moe && kTensor && HH % 16 == 0) {
      // ---- gate logits of hx_moe / x_moe (:56) on clamp(o): [tokens x HH] @ [HH x 2r] on
      // mma.sync, a warp per 8 gate rows, rounded to the dtype
      const int g = lane >> 2, c = lane & 3;
      for (int nt = warp; nt < 2 * r / 8; nt += nw) {
        const int ri = (nt * 8) / r, j0 = nt * 8 - ri * r;
        const T* Wr = L.staged ? reinterpret_cast<const T*>(smb + L.g16) + (size_t)ri * r * HH
                               : reinterpret_cast<const T*>(p.rt[ri].gate_w);
        const T* W = Wr + (size_t)(j0 + g) * HH + 2 * c;
        const float* xs = g < ntok ? reinterpret_cast<const float*>(smb + L.tok0 + g * L.tk.bytes + L.tk.xs) : nullptr;
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        for (int ks = 0; ks < HH; ks += 16) {
          uint32_t a[4] = {0u, 0u, 0u, 0u};
          if (xs) {
            a[0] = pack_bf16(xs[ks + 2 * c], xs[ks + 2 * c + 1]);
            a[2] = pack_bf16(xs[ks + 2 * c + 8], xs[ks + 2 * c + 9]);
          }
          mma_16816_bf16(acc, a, ldg_u32(W + ks), ldg_u32(W + ks + 8));
        }
        if (xs) {
          float* gl = reinterpret_cast<float*>(smb + L.tok0 + g * L.tk.bytes + L.tk.gl) + ri * r;
          gl[j0 + 2 * c] = rnd<T>(acc[0]);
          gl[j0 + 2 * c + 1] = rnd<T>(acc[1]);
        }
      }
      __syncthreads();
    }
    if (p.use_moe) {
      // ---- phase B: routers, warps grouped per token slot (6 warps each)
      const int k = warp / 6, role = warp % 6;
      if (k < ntok && warp < 6 * kAttnTok) {
        const int t = t0 + k;
        uint8_t* tb = smb + L.tok0 + k * L.tk.bytes;
        const float* xs = reinterpret_cast<const float*>(tb + L.tk.xs);
        const float* cxs = reinterpret_cast<const float*>(tb + L.tk.cxs);
        float* gl = reinterpret_cast<float*>(tb + L.tk.gl);
        float* cvb = reinterpret_cast<float*>(tb + L.tk.cv);
        double* part = reinterpret_cast<double*>(tb + L.tk.part);
        float* sc = reinterpret_cast<float*>(tb + L.tk.sc);
        int* sel = reinterpret_cast<int*>(tb + L.tk.sel);
        const int kk = min(p.k, E);
        if (role < 2) {
          // hx_moe (role 0) / x_moe (role 1) on clamp(o)
          const int ri = role;
          float* g = gl + ri * r;
          const T* Wg = reinterpret_cast<const T*>(p.rt[ri].gate_w);
          for (int j = lane; j < r && !(kTensor && HH % 16 == 0); j += 32) {
            const T* wr = Wg + j * HH;
            float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
            int i = 0;
#pragma unroll 2
            for (; i + 4 <= HH; i += 4) {
              a0 = fmaf(ld<T>(wr + i), xs[i], a0);
              a1 = fmaf(ld<T>(wr + i + 1), xs[i + 1], a1);
              a2 = fmaf(ld<T>(wr + i + 2), xs[i + 2], a2);
              a3 = fmaf(ld<T>(wr + i + 3), xs[i + 3], a3);
            }
            for (; i < HH; ++i) a0 = fmaf(ld<T>(wr + i), xs[i], a0);
            g[j] = rnd<T>((a0 + a1) + (a2 + a3));  // gate logits (:56)
          }
          __syncwarp();
          float* c = cvb + ri * E;
          double* cp = reinterpret_cast<double*>(tb + L.tk.scr) + role * 32;
          warp_gate_factors<T>(g, r, exps + ri * E, E, c, cp);
          const T* B2 = b2s + b2off[ri];
          for (int e0 = 0; e0 < E; e0 += 8) {
            const double tot = warp_expert_sums_t<T>(xs, 0, HH, B2, HH, c, e0, E);
            const int sl = e0 + r2_slot(lane);
            if ((lane & 3) == 0 && sl < E) sc[ri * E + sl] = rnd<T>(__double2float_rn(tot));
          }
          __syncwarp();
          if (lane == 0) {
            int chosen[kMaxExperts];
            topk_select_fast(sc + ri * E, E, kk, chosen, p.tie);
            for (int j = 0; j < kk; ++j) {
              sel[ri * E + j] = chosen[j];
              if (p.rt[ri].idx_out) p.rt[ri].idx_out[(size_t)t * kk + j] = chosen[j];
            }
          }
          __syncwarp();
          warp_combine<T>(xs, 0, HH, B2, HH, c, sel + ri * E, kk, reinterpret_cast<T*>(p.rt[ri].comb) + (size_t)t * HH);
        } else {
          // cx_moe on clamp(cx): four warps, each a quarter of the inputs
          const int q = role - 2;
          const int bar = 1 + k;
          float* g = gl + 2 * r;
          float* c = cvb + (2 + q) * E;
          // each warp normalises its own copy of the gate logits
          float* gg = reinterpret_cast<float*>(tb + L.tk.gq) + q * r;
          for (int j = lane; j < r; j += 32) gg[j] = g[j];
          __syncwarp();
          warp_gate_factors<T>(gg, r, exps + 2 * E, E, c, reinterpret_cast<double*>(tb + L.tk.scr) + role * 32);
          const int qlen = (D + kAttnCxWarps - 1) / kAttnCxWarps;
          const int i0 = q * qlen, i1 = min(D, i0 + qlen);
          const T* B2 = b2s + b2off[2];
          for (int e0 = 0; e0 < E; e0 += 8) {
            const double tot = warp_expert_sums_t<T>(cxs, i0, i1, B2, D, c, e0, E);
            const int sl = e0 + r2_slot(lane);
            if ((lane & 3) == 0 && sl < E) part[q * kMaxExperts + sl] = tot;
          }
          named_bar(bar, 32 * kAttnCxWarps);
          if (q == 0) {
            for (int e = lane; e < E; e += 32) {  // the quarters' partials added in quarter order
              double s2 = 0.0;
              for (int qq = 0; qq < kAttnCxWarps; ++qq) s2 += part[qq * kMaxExperts + e];
              sc[2 * E + e] = rnd<T>(__double2float_rn(s2));
            }
            __syncwarp();
            if (lane == 0) {
              int chosen[kMaxExperts];
              topk_select_fast(sc + 2 * E, E, kk, chosen, p.tie);
              for (int j = 0; j < kk; ++j) {
                sel[2 * E + j] = chosen[j];
                if (p.rt[2].idx_out) p.rt[2].idx_out[(size_t)t * kk + j] = chosen[j];
              }
            }
          }
          named_bar(bar, 32 * kAttnCxWarps);
          warp_combine<T>(cxs, i0, i1, B2, D, c, sel + 2 * E, kk, reinterpret_cast<T*>(p.rt[2].comb) + (size_t)t * D);
        }
      }
    }
    __syncthreads();
  }
}

// Standalone LinearMoE router (one/linear_moe.py:53-90) on precomputed gate logits, with the
// same steps and rounding as the decode path's routers (warp_gate_factors, warp_expert_sums,
// topk_select, warp_combine). Each warp takes groups of `group` (<= 32) tokens: for every token of
// the group it computes the expert factors and scores; then the group's selections run
// side by side, one token per lane (the selection is a sequential algorithm whose output
// order matters, so it is parallelised across tokens, not within one); then each token's
// biased inputs are combined. bias2 (when it fits) and the clamped experts are staged once
// per CTA; per warp: one token's clamped input and gate values, and the group's factors,
// scores and selections.
constexpr size_t kRouterStageB2Max = 48 * 1024;
struct RouterSmem {
  size_t b2, ex, warp0, per_warp, total, xs, g, cf, sc, sel;
  int warps;
  bool stage_b2;
};
__host__ __device__ inline RouterSmem router_smem(int in, int r, int E, int es) {
  RouterSmem L;
  const size_t b2 = (size_t)E * in * es;
  L.stage_b2 = b2 <= kRouterStageB2Max;
  L.b2 = 0;
  L.ex = (L.stage_b2 ? (b2 + 15) & ~size_t(15) : 0);
  // per warp: 32 doubles of scratch, x [in], gate [r], group factors / scores / selections [32][E]
  L.xs = 256;
  L.g = L.xs + (size_t)in * 4;
  L.cf = L.g + (size_t)r * 4;
  L.sc = L.cf + (size_t)32 * E * 4;
  L.sel = L.sc + (size_t)32 * E * 4;
  L.per_warp = (L.sel + (size_t)32 * E * 4 + 15) & ~size_t(15);
  L.warp0 = L.ex + (size_t)kMaxExperts * 4;
  const size_t budget = 200 * 1024 - L.warp0;
  L.warps = (int)(budget / L.per_warp < 8 ? budget / L.per_warp : 8);
  L.total = L.warp0 + (size_t)(L.warps > 0 ? L.warps : 1) * L.per_warp;
  return L;
}

template <typename T>
__global__ void __launch_bounds__(256) moe_router_kernel(const MoeRouter R, int ntok, int r, int E, int k, int group,
                                                         unsigned long long tie) {
  extern __shared__ __align__(16) uint8_t rsm[];
  const int in = R.in, lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarp = blockDim.x >> 5;
  const RouterSmem L = router_smem(in, r, E, (int)sizeof(T));
  float* ex = reinterpret_cast<float*>(rsm + L.ex);
  uint8_t* wb = rsm + L.warp0 + warp * L.per_warp;
  double* cp = reinterpret_cast<double*>(wb);
  float* xs = reinterpret_cast<float*>(wb + L.xs);
  float* g = reinterpret_cast<float*>(wb + L.g);
  float* cf = reinterpret_cast<float*>(wb + L.cf);  // [32][E] expert factors of the group
  float* sc = reinterpret_cast<float*>(wb + L.sc);  // [32][E] expert scores
  int* sel = reinterpret_cast<int*>(wb + L.sel);    // [32][E] chosen experts
  pdl_wait();
  const T* B2 = reinterpret_cast<const T*>(R.bias2);
  if (L.stage_b2) {
    constexpr int VE = 16 / (int)sizeof(T);
    T* b2s = reinterpret_cast<T*>(rsm + L.b2);
    const int nv = E * in / VE;
    if ((E * in) % VE == 0 && (reinterpret_cast<uintptr_t>(B2) & 15) == 0)
      for (int v = threadIdx.x; v < nv; v += blockDim.x)
        reinterpret_cast<uint4*>(b2s)[v] = reinterpret_cast<const uint4*>(B2)[v];
    else
      for (int v = threadIdx.x; v < E * in; v += blockDim.x) b2s[v] = B2[v];
    B2 = b2s;
  }
  for (int e = threadIdx.x; e < E; e += blockDim.x)
    ex[e] = fminf(fmaxf(ld<T>(reinterpret_cast<const T*>(R.experts) + e), -10.f), 10.f);
  __syncthreads();
  const int kk = min(k, E);
  auto load_x = [&](int t) {
    const T* X = reinterpret_cast<const T*>(R.x) + (size_t)t * R.ldx;
    for (int i = lane; i < in; i += 32) xs[i] = moe_clamp<T>(ld<T>(X + i));  // (:53)
  };
  group = max(1, min(32, group));
  for (int t0 = (blockIdx.x * nwarp + warp) * group; t0 < ntok; t0 += gridDim.x * nwarp * group) {
    const int nt = min(group, ntok - t0);
    for (int u = 0; u < nt; ++u) {
      const int t = t0 + u;
      load_x(t);
      const T* G = reinterpret_cast<const T*>(R.glog) + (size_t)t * r;
      for (int j = lane; j < r; j += 32) g[j] = ld<T>(G + j);
      __syncwarp();
      float* c = cf + u * E;
      warp_gate_factors<T>(g, r, ex, E, c, cp);  // softmax (:56), expert factors (:59-68)
      for (int e0 = 0; e0 < E; e0 += 8) {        // exact per-expert sums (:71-80)
        const double tot = warp_expert_sums_t<T>(xs, 0, in, B2, in, c, e0, E);
        const int sl = e0 + r2_slot(lane);
        if ((lane & 3) == 0 && sl < E) sc[u * E + sl] = rnd<T>(__double2float_rn(tot));
      }
      __syncwarp();
    }
    if (lane < nt) {  // top-k (:83-84), one token per lane
      topk_select_fast(sc + lane * E, E, kk, sel + lane * E, tie);
      if (R.idx_out)
        for (int j = 0; j < kk; ++j) R.idx_out[(size_t)(t0 + lane) * kk + j] = sel[lane * E + j];
    }
    __syncwarp();
    for (int u = 0; u < nt; ++u) {  // mean of the chosen biased inputs (:87-90)
      load_x(t0 + u);
      __syncwarp();
      warp_combine<T>(xs, 0, in, B2, in, cf + u * E, sel + u * E, kk,
                      reinterpret_cast<T*>(R.comb) + (size_t)(t0 + u) * in);
      __syncwarp();
    }
  }
}

inline size_t moe_router_smem_bytes(int in, int r, int E, int es) { return router_smem(in, r, E, es).total; }
inline int moe_router_warps(int in, int r, int E, int es) { return router_smem(in, r, E, es).warps; }


}  // namespace one
