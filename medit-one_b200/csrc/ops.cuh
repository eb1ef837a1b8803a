// Standalone operators behind the legacy one_turbo entry points.
#pragma once

#include "common.cuh"

namespace one {

// OneRotaryEmbedding.forward (one/modeling_one.py:159-182): freqs = inv_freq * pos in
// fp32, emb = cat(freqs, freqs), cos / sin cast to the output dtype.
template <typename T>
__global__ void rotary_kernel(const int64_t* pos, int n, const float* inv_freq, int dim, T* cos_out, T* sin_out) {
  pdl_wait();  // launched with programmatic stream serialization: inputs visible after this
  const int half = dim / 2;
  const long idx = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (long)n * half) return;
  const int row = (int)(idx / half), i = (int)(idx % half);
  const float f = inv_freq[i] * (float)pos[row];
  const float c = cosf(f), s = sinf(f);
  st<T>(cos_out + (size_t)row * dim + i, c);
  st<T>(cos_out + (size_t)row * dim + i + half, c);
  st<T>(sin_out + (size_t)row * dim + i, s);
  st<T>(sin_out + (size_t)row * dim + i + half, s);
}

// turbo_cumsum_and_normalize_cpu (one/turbo_ops.py:288-310): fp32 prefix sum along s,
// divided by (s + 1 + 1e-8) in fp32, cast back. One thread per (batch, feature).
template <typename T>
__global__ void cumsum_norm_kernel(const T* x, int b, int s, int d, int seq_len, T* out) {
  pdl_wait();  // launched with programmatic stream serialization: inputs visible after this
  const long idx = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (long)b * d) return;
  const int bb = (int)(idx / d), j = (int)(idx % d);
  float acc = 0.f;
  const int n = min(s, seq_len);
  for (int t = 0; t < n; ++t) {
    acc += ld<T>(x + ((size_t)bb * s + t) * d + j);
    st<T>(out + ((size_t)bb * n + t) * d + j, acc / ((float)(t + 1) + 1e-8f));
  }
}

// The model's feature attention (one/modeling_one.py:515-547) on [b, h, t, dh] inputs:
// RoPE, three dh -> hout projections with bias, softmax(q*k - max) in fp32, times v.
// One thread per (b, h, t) row.
template <typename T>
__global__ void combined_rope_attn_kernel(const T* sx, const T* ky, const T* va, const T* cosv, const T* sinv, int cos_b,
                                          const T* wq, const T* bq, const T* wk, const T* bk, const T* wv, const T* bv,
                                          int b, int h, int t, int dh, int hout, T* out) {
  pdl_wait();  // launched with programmatic stream serialization: inputs visible after this
  const long idx = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (long)b * h * t) return;
  const int ti = (int)(idx % t);
  const int bi = (int)(idx / ((long)h * t));
  const int half = dh / 2;
  const T* X = sx + idx * dh;
  const T* K = ky + idx * dh;
  const T* V = va + idx * dh;
  const int cb = cos_b > 1 ? bi : 0;
  const T* C = cosv + ((size_t)cb * t + ti) * dh;
  const T* S = sinv + ((size_t)cb * t + ti) * dh;
  float q[64], k[64], v[64];
  for (int o = 0; o < hout; ++o) {
    float aq = 0.f, ak = 0.f, av = 0.f;
    for (int i = 0; i < dh; ++i) {
      const float c = ld<T>(C + i), s = ld<T>(S + i);
      const float xi = ld<T>(X + i), ki = ld<T>(K + i);
      const float xp = i < half ? -ld<T>(X + i + half) : ld<T>(X + i - half);
      const float kp = i < half ? -ld<T>(K + i + half) : ld<T>(K + i - half);
      const float xr = rnd<T>(rnd<T>(xi * c) + rnd<T>(xp * s));
      const float kr = rnd<T>(rnd<T>(ki * c) + rnd<T>(kp * s));
      aq = fmaf(ld<T>(wq + o * dh + i), xr, aq);
      ak = fmaf(ld<T>(wk + o * dh + i), kr, ak);
      av = fmaf(ld<T>(wv + o * dh + i), ld<T>(V + i), av);
    }
    q[o] = rnd<T>(aq + (bq ? ld<T>(bq + o) : 0.f));
    k[o] = rnd<T>(ak + (bk ? ld<T>(bk + o) : 0.f));
    v[o] = rnd<T>(av + (bv ? ld<T>(bv + o) : 0.f));
  }
  float mx = -INFINITY;
  for (int o = 0; o < hout; ++o) {
    q[o] = rnd<T>(q[o] * k[o]);
    mx = fmaxf(mx, q[o]);
  }
  float m2 = -INFINITY;
  for (int o = 0; o < hout; ++o) {
    q[o] = rnd<T>(q[o] - mx);
    m2 = fmaxf(m2, q[o]);
  }
  float sum = 0.f;
  for (int o = 0; o < hout; ++o) {
    q[o] = expf(q[o] - m2);
    sum += q[o];
  }
  const float inv = 1.0f / sum;
  T* O = out + idx * hout;
  for (int o = 0; o < hout; ++o) {
    float w = q[o] * inv;
    w = isnan(w) ? 1.0f / (float)hout : rnd<T>(w);
    st<T>(O + o, w * v[o]);
  }
}

// Exact softmax attention (turbo_flash_attention's PyTorch path, one/turbo_ops.py:
// 115-143) on CUDA cores: q scaled and rounded, scores rounded to the dtype, fp32 online
// softmax, output rounded once. One thread per query row, 64-key tiles in shared memory.
template <typename T>
__global__ void __launch_bounds__(64) attn_simt_kernel(const T* q, const T* k, const T* v, int nq, int nk, int dh,
                                                       int causal, float scale, T* out) {
  pdl_wait();  // launched with programmatic stream serialization: inputs visible after this
  __shared__ float sK[64][65];
  __shared__ float sV[64][65];
  const int bh = blockIdx.y;
  const int row = blockIdx.x * 64 + threadIdx.x;
  const T* Q = q + ((size_t)bh * nq + min(row, nq - 1)) * dh;
  float qr[64], acc[64];
  for (int i = 0; i < dh; ++i) {
    qr[i] = rnd<T>(ld<T>(Q + i) * scale);
    acc[i] = 0.f;
  }
  float m = -INFINITY, l = 0.f;
  const int kend = causal ? min(nk, blockIdx.x * 64 + 64) : nk;
  for (int k0 = 0; k0 < kend; k0 += 64) {
    __syncthreads();
    for (int i = threadIdx.x; i < 64 * dh; i += 64) {
      const int r = i / dh, c = i % dh;
      const bool ok = k0 + r < nk;
      sK[r][c] = ok ? ld<T>(k + ((size_t)bh * nk + k0 + r) * dh + c) : 0.f;
      sV[r][c] = ok ? ld<T>(v + ((size_t)bh * nk + k0 + r) * dh + c) : 0.f;
    }
    __syncthreads();
    const int kn = min(64, nk - k0);
    for (int j = 0; j < kn; ++j) {
      if (causal && k0 + j > row) break;
      float s = 0.f;
      for (int i = 0; i < dh; ++i) s = fmaf(qr[i], sK[j][i], s);
      s = rnd<T>(s);
      const float mn = fmaxf(m, s);
      const float corr = expf(m - mn);
      const float pj = expf(s - mn);
      l = l * corr + pj;
      for (int i = 0; i < dh; ++i) acc[i] = acc[i] * corr + pj * sV[j][i];
      m = mn;
    }
  }
  if (row < nq) {
    T* O = out + ((size_t)bh * nq + row) * dh;
    for (int i = 0; i < dh; ++i) st<T>(O + i, acc[i] / l);
  }
}

}  // namespace one
