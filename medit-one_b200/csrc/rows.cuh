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
  // previous layer's tail
  const float* ws;        // [splits][T][D] down_proj partials
  int splits;
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

template <typename T, int NV>
__global__ void __launch_bounds__(256) row_pre_kernel(const RowPreParams p) {
  pdl_wait();
  const int warps = blockDim.x >> 5;
  const int t = blockIdx.x * warps + (threadIdx.x >> 5);
  if (t >= p.T) return;
  const int lane = threadIdx.x & 31;
  const int D = p.D, nch = D / 8;
  const size_t row = (size_t)t * D;
  float h[NV][8], a[NV][8], b[NV][8];

  if (p.mode == PRE_FIRST) {
    int id;
    if (p.ids_from_best) {
      const unsigned long long key = p.best[t];
      id = key ? (int)(0xFFFFFFFFu - (uint32_t)(key & 0xFFFFFFFFull)) : 0;
    } else {
      id = p.ids[t];
    }
    if (id < 0 || id >= p.vocab) {  // never gather outside the embedding table
      if (lane == 0) set_err(p.err, ERR_BAD_ARG, 100);
      id = 0;
    }
    __syncwarp();
    if (lane == 0) {
      // this step's lm_head argmax accumulates into best[t] again
      p.best[t] = 0ull;
      if (p.ids_out) p.ids_out[t] = id;
      if (p.hist) {
        const int step = p.counters[1];
        if (step < p.hist_cap) p.hist[(size_t)step * p.T + t] = id;
      }
    }
    warp_load_row<T, NV>(reinterpret_cast<const T*>(p.emb) + (size_t)id * D, nch, h);
#pragma unroll
    for (int j = 0; j < NV; ++j)
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        a[j][e] = 1.0f;
        b[j][e] = fminf(fmaxf(h[j][e], -1e4f), 1e4f);
      }
    warp_store_row<T, NV>(reinterpret_cast<T*>(p.hx) + row, nch, a);
    warp_store_row<T, NV>(reinterpret_cast<T*>(p.cx) + row, nch, h);
    warp_store_row<T, NV>(reinterpret_cast<T*>(p.cxc) + row, nch, b);
  } else {
    // finish the previous layer: out = norm(out0 + down_proj(...)) (:571-573), h += out (:793)
    warp_load_row<T, NV>(reinterpret_cast<const T*>(p.out0) + row, nch, a);
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int c = lane + 32 * j;
      if (c < nch) {
        float m[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int s = 0; s < p.splits; ++s) {
          float v[8];
          load8(p.ws + ((size_t)s * p.T + t) * D + c * 8, v);
#pragma unroll
          for (int e = 0; e < 8; ++e) m[e] += v[e];
        }
        if (p.down_b) {
          float v[8];
          load8(reinterpret_cast<const T*>(p.down_b) + c * 8, v);
#pragma unroll
          for (int e = 0; e < 8; ++e) m[e] += v[e];
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) a[j][e] = rnd<T>(a[j][e] + rnd<T>(m[e]));
      }
    }
    const T* nw = reinterpret_cast<const T*>(p.prev_norm_w);
    const T* nb = reinterpret_cast<const T*>(p.prev_norm_b);
    warp_rmsnorm<T, NV>(a, nch, nw, nb, 1e-6f, D, b);
    warp_load_row<T, NV>(reinterpret_cast<const T*>(p.h) + row, nch, h);
#pragma unroll
    for (int j = 0; j < NV; ++j)
#pragma unroll
      for (int e = 0; e < 8; ++e) h[j][e] = rnd<T>(h[j][e] + b[j][e]);
    // hx = norm(hx + hx_moe) (:563-564)
    warp_load_row<T, NV>(reinterpret_cast<const T*>(p.hx_pre) + row, nch, a);
    warp_rmsnorm<T, NV>(a, nch, nw, nb, 1e-6f, D, b);
    warp_store_row<T, NV>(reinterpret_cast<T*>(p.hx) + row, nch, b);
    if (p.mode == PRE_FINAL) {
      warp_store_row<T, NV>(reinterpret_cast<T*>(p.h) + row, nch, h);
      warp_rmsnorm<T, NV>(h, nch, reinterpret_cast<const T*>(p.lhs_w), reinterpret_cast<const T*>(p.lhs_b), p.lhs_eps, D, a);
      warp_store_row<T, NV>(reinterpret_cast<T*>(p.hf) + row, nch, a);
      return;
    }
  }
  warp_store_row<T, NV>(reinterpret_cast<T*>(p.h) + row, nch, h);
  // norm_x = norm1(h) (:340); OneRMSNorm(dim) keeps eps = 1e-6 and has no bias
  warp_rmsnorm<T, NV>(h, nch, reinterpret_cast<const T*>(p.norm1_w), (const T*)nullptr, 1e-6f, D, a);
  warp_store_row<T, NV>(reinterpret_cast<T*>(p.norm_x) + row, nch, a);
  if (p.decode) {
    // running sum replaces cache.update + cumsum (:358-376); mean = sum / arange[-1] (:379-387)
    const float dv = p.div[p.counters[0]];
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int c = lane + 32 * j;
      if (c < nch) {
        float s[8];
        load8(p.S + row + c * 8, s);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          s[e] += a[j][e];
          b[j][e] = rnd<T>(rnd<T>(s[e]) / dv);
        }
        store8(p.S + row + c * 8, s);
      }
    }
    warp_store_row<T, NV>(reinterpret_cast<T*>(p.mean) + row, nch, b);
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
};

template <typename T>
__global__ void __launch_bounds__(256) scan_mean_kernel(const ScanParams p) {
  pdl_wait();
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= p.B * p.D) return;
  const int bb = idx / p.D, d = idx % p.D;
  float acc = p.state[idx];
  const T* x = reinterpret_cast<const T*>(p.norm_x) + (size_t)bb * p.S * p.D + d;
  T* m = reinterpret_cast<T*>(p.mean) + (size_t)bb * p.S * p.D + d;
  for (int s = 0; s < p.S; ++s) {
    acc += ld<T>(x + (size_t)s * p.D);
    st<T>(m + (size_t)s * p.D, rnd<T>(acc) / p.div[s]);
  }
  p.state[idx] = acc;
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
  DevErr* err;
};

// One LinearMoE router for one token (one/linear_moe.py:53-90), executed by the CTA.
// xs: router input in shared memory (fp32 values of model-dtype numbers).
template <typename T>
__device__ void cta_router(int r, int E, int k, const MoeRouter& R, int t, const float* xs, float* gl, float* cvals,
                           double* red, float* score, int* sel) {
  const int tid = threadIdx.x, nt = blockDim.x;
  const int in = R.in;
  // gate logits (:56)
  if (R.gate_w) {
    const T* W = reinterpret_cast<const T*>(R.gate_w);
    for (int j = tid; j < r; j += nt) {
      float acc = 0.f;
      const T* wr = W + (size_t)j * in;
      for (int i = 0; i < in; ++i) acc = fmaf(ld<T>(wr + i), xs[i], acc);
      gl[j] = rnd<T>(acc);
    }
  } else {
    const T* G = reinterpret_cast<const T*>(R.glog) + (size_t)t * r;
    for (int j = tid; j < r; j += nt) gl[j] = ld<T>(G + j);
  }
  __syncthreads();
  // softmax over r in fp32 (:56), expert scores (:59-68): one warp per expert
  if (tid < 32) {
    float mx = -INFINITY;
    for (int j = tid; j < r; j += 32) mx = fmaxf(mx, gl[j]);
    mx = warp_max(mx);
    float sum = 0.f;
    for (int j = tid; j < r; j += 32) sum += expf(gl[j] - mx);
    sum = warp_sum(sum);
    const float inv = 1.0f / sum;
    __syncwarp();
    for (int j = tid; j < r; j += 32) gl[j] = rnd<T>(expf(gl[j] - mx) * inv);
  }
  __syncthreads();
  const T* EX = reinterpret_cast<const T*>(R.experts);
  for (int e = tid; e < E; e += nt) {
    const float ex = fminf(fmaxf(ld<T>(EX + e), -10.f), 10.f);
    float s = 0.f;
    for (int j = 0; j < r; ++j) s += rnd<T>(gl[j] * ex);   // fp32 sum in r order, then / r
    float sc = fminf(fmaxf(rnd<T>(s / (float)r), -10.f), 10.f);
    cvals[e] = rnd<T>(1.0f + rnd<T>(silu_f(sc)));
  }
  __syncthreads();
  // per-expert sums of x * c_e + bias2[e] (:71-80): exact (fp64) sum, rounded once
  const T* B2 = reinterpret_cast<const T*>(R.bias2);
  for (int e0 = 0; e0 < E; e0 += 8) {
    double acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int i = tid; i < in; i += nt) {
#pragma unroll
      for (int e = 0; e < 8; ++e)
        if (e0 + e < E) acc[e] += (double)rnd<T>(rnd<T>(xs[i] * cvals[e0 + e]) + ld<T>(B2 + (size_t)(e0 + e) * in + i));
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = warp_sum_d(acc[e]);
    const int w = tid >> 5, lane = tid & 31;
    if (lane == 0)
#pragma unroll
      for (int e = 0; e < 8; ++e) red[w * 8 + e] = acc[e];
    __syncthreads();
    if (tid < 8 && e0 + tid < E) {
      double s = 0.0;
      for (int ww = 0; ww < (nt >> 5); ++ww) s += red[ww * 8 + tid];
      score[e0 + tid] = rnd<T>(__double2float_rn(s));
    }
    __syncthreads();
  }
  if (tid == 0) {
    const int kk = min(k, E);
    topk_select(score, E, kk, sel);
    if (R.idx_out)
      for (int j = 0; j < kk; ++j) R.idx_out[(size_t)t * kk + j] = sel[j];
  }
  __syncthreads();
  // mean of the selected biased inputs (:87-90), fp32 sum in selection order
  const int kk = min(k, E);
  T* C = reinterpret_cast<T*>(R.comb) + (size_t)t * in;
  for (int i = tid; i < in; i += nt) {
    float s = 0.f;
    for (int j = 0; j < kk; ++j) {
      const int e = sel[j];
      s += rnd<T>(rnd<T>(xs[i] * cvals[e]) + ld<T>(B2 + (size_t)e * in + i));
    }
    st<T>(C + i, s / (float)kk);
  }
  __syncthreads();
}

// Feature attention (one/modeling_one.py:390-556): per head, RoPE on single_x * scale
// and on key, three Dh->H projections, softmax(q*k - max) in fp32, times v; then the
// hx_moe / x_moe routers on the H*H outputs and the cx_moe router on cx.
template <typename T>
__global__ void __launch_bounds__(128) row_attn_kernel(const RowAttnParams p) {
  extern __shared__ float sm[];
  const int H = p.H, Dh = p.Dh, HD = H * Dh, HH = H * H;
  float* sx = sm;                 // [HD] single_x * scale
  float* sk = sx + HD;            // [HD] key
  float* sv = sk + HD;            // [HD] value
  float* sxr = sv + HD;           // [HD] RoPE(single_x)
  float* skr = sxr + HD;          // [HD] RoPE(key)
  float* qkv = skr + HD;          // [3][HH]
  float* so = qkv + 3 * HH;       // [HH]
  float* cs = so + HH;            // [Dh] cos, [Dh] sin
  float* gl = cs + 2 * Dh;        // [r]
  float* cvals = gl + p.r;        // [E]
  float* score = cvals + kMaxExperts;     // [E]
  float* xs = score + kMaxExperts;        // router input, up to max(HH, D)
  int* sel = reinterpret_cast<int*>(xs + 4096);
  double* red = reinterpret_cast<double*>((reinterpret_cast<uintptr_t>(sel + kMaxExperts) + 7) & ~uintptr_t(7));  // [warps*8]
  pdl_wait();
  const int tid = threadIdx.x, nt = blockDim.x;
  const int half = Dh / 2;
  for (int t = blockIdx.x; t < p.T; t += gridDim.x) {
    const int pos = p.counters[0] + (p.seq_len > 0 ? t % p.seq_len : 0);
    // cos/sin (OneRotaryEmbedding, :159-182): fp32 freq = inv_freq * pos, cast to dtype
    for (int i = tid; i < half; i += nt) {
      const float f = p.inv_freq[i] * (float)pos;
      const float c = rnd<T>(cosf(f)), s = rnd<T>(sinf(f));
      cs[i] = c; cs[i + half] = c;
      cs[Dh + i] = s; cs[Dh + i + half] = s;
    }
    const T* pr = reinterpret_cast<const T*>(p.proj) + (size_t)t * 3 * HD;
    for (int i = tid; i < HD; i += nt) {
      sx[i] = rnd<T>(ld<T>(pr + i) * p.attn_scale);  // :405
      sk[i] = ld<T>(pr + HD + i);
      sv[i] = ld<T>(pr + 2 * HD + i);
    }
    __syncthreads();
    // rotate_half RoPE (one/flash_attention.py:20-33): x*cos + rotate_half(x)*sin
    for (int i = tid; i < HD; i += nt) {
      const int d = i % Dh, base = i - d;
      const float px = d < half ? -sx[base + d + half] : sx[base + d - half];
      const float pk = d < half ? -sk[base + d + half] : sk[base + d - half];
      sxr[i] = rnd<T>(rnd<T>(sx[i] * cs[d]) + rnd<T>(px * cs[Dh + d]));
      skr[i] = rnd<T>(rnd<T>(sk[i] * cs[d]) + rnd<T>(pk * cs[Dh + d]));
    }
    __syncthreads();
    // q = lin_q(xr), k = lin_k(kr), v = lin_v(value): Dh -> H per head, with bias
    for (int w = tid; w < 3 * HH; w += nt) {
      const int which = w / HH, hj = w % HH, h = hj / H, j = hj % H;
      const T* W = reinterpret_cast<const T*>(which == 0 ? p.wq : which == 1 ? p.wk : p.wv);
      const T* Bb = reinterpret_cast<const T*>(which == 0 ? p.bq : which == 1 ? p.bk : p.bv);
      const float* src = (which == 0 ? sxr : which == 1 ? skr : sv) + h * Dh;
      float acc = 0.f;
      for (int d = 0; d < Dh; ++d) acc = fmaf(ld<T>(W + j * Dh + d), src[d], acc);
      qkv[which * HH + hj] = rnd<T>(acc + ld<T>(Bb + j));
    }
    __syncthreads();
    // softmax(q*k - max) in fp32, cast, NaN -> 1/H, times v (:530-547)
    for (int h = tid; h < H; h += nt) {
      float lg[64];
      float mx = -INFINITY;
      for (int j = 0; j < H; ++j) {
        lg[j] = rnd<T>(qkv[h * H + j] * qkv[HH + h * H + j]);
        mx = fmaxf(mx, lg[j]);
      }
      float m2 = -INFINITY;
      for (int j = 0; j < H; ++j) {
        lg[j] = rnd<T>(lg[j] - mx);
        m2 = fmaxf(m2, lg[j]);
      }
      float sum = 0.f;
      for (int j = 0; j < H; ++j) {
        lg[j] = expf(lg[j] - m2);
        sum += lg[j];
      }
      const float inv = 1.0f / sum;
      for (int j = 0; j < H; ++j) {
        float w = lg[j] * inv;
        w = isnan(w) ? 1.0f / (float)H : rnd<T>(w);
        so[h * H + j] = rnd<T>(w * qkv[2 * HH + h * H + j]);
      }
    }
    __syncthreads();
    if (p.o) {
      T* O = reinterpret_cast<T*>(p.o) + (size_t)t * HH;
      for (int i = tid; i < HH; i += nt) st<T>(O + i, so[i]);
    }
    if (p.use_moe) {
      // hx_moe and x_moe route the same attention output, clamped to +-1e4 (:53)
      for (int i = tid; i < HH; i += nt) xs[i] = fminf(fmaxf(so[i], -1e4f), 1e4f);
      __syncthreads();
      cta_router<T>(p.r, p.E, p.k, p.rt[0], t, xs, gl, cvals, red, score, sel);
      cta_router<T>(p.r, p.E, p.k, p.rt[1], t, xs, gl, cvals, red, score, sel);
      // cx_moe routes clamp(cx), with gate logits from the projection GEMM
      const MoeRouter& R = p.rt[2];
      const T* X = reinterpret_cast<const T*>(R.x) + (size_t)t * R.ldx;
      for (int i = tid; i < R.in; i += nt) xs[i] = ld<T>(X + i);
      __syncthreads();
      cta_router<T>(p.r, p.E, p.k, R, t, xs, gl, cvals, red, score, sel);
    }
    __syncthreads();
  }
}


// LinearMoE router alone (standalone op): per token, clamp the input (:53), then the
// router of cta_router. gate logits come precomputed in R.glog.
template <typename T>
__global__ void __launch_bounds__(128) moe_router_kernel(const MoeRouter R, int ntok, int r, int E, int k) {
  extern __shared__ float sm[];
  float* xs = sm;                   // [in]
  float* gl = xs + R.in;            // [r]
  float* cvals = gl + r;            // [E]
  float* score = cvals + kMaxExperts;
  int* sel = reinterpret_cast<int*>(score + kMaxExperts);
  double* red = reinterpret_cast<double*>((reinterpret_cast<uintptr_t>(sel + kMaxExperts) + 7) & ~uintptr_t(7));
  pdl_wait();
  for (int t = blockIdx.x; t < ntok; t += gridDim.x) {
    const T* X = reinterpret_cast<const T*>(R.x) + (size_t)t * R.ldx;
    for (int i = threadIdx.x; i < R.in; i += blockDim.x) xs[i] = fminf(fmaxf(ld<T>(X + i), -1e4f), 1e4f);
    __syncthreads();
    cta_router<T>(r, E, k, R, t, xs, gl, cvals, red, score, sel);
  }
}

inline size_t moe_router_smem_bytes(int in, int r) {
  return (size_t)(in + r + 2 * kMaxExperts) * 4 + (kMaxExperts + 2) * 4 + 8 + 4 * 8 * 8;
}

inline size_t row_attn_smem_bytes(int H, int Dh, int r) {
  const int HD = H * Dh, HH = H * H;
  size_t f = (size_t)5 * HD + 4 * HH + 2 * Dh + r + 2 * kMaxExperts + 4096;
  size_t bytes = f * 4 + kMaxExperts * 4;
  bytes = (bytes + 7) & ~(size_t)7;
  return bytes + 8 + 4 * 8 * 8;  // align slack + warps * 8 doubles
}

}  // namespace one
