// Decode-step feature attention and the three LinearMoE routers (bf16, LinearMoE layers,
// H <= 16 even, head_dim 32 / 64, r <= 128 and a multiple of 16, H*H a multiple of 16),
// two tokens per CTA with the work split by warp so that independent chains overlap:
//
//   warps 0, 1   token 0 / 1: attention (attn_token_warp: RoPE, lin_q / lin_k / lin_v on
//                mma.sync with the heads as rows, softmax, o = w * v, LinearMoE clamp), then
//                a quarter of the hx_moe / x_moe gate logits of both tokens (CUDA cores), then
//                the hx_moe / x_moe router of token 0
//   warps 10, 11 the step position's cos / sin (while the rows load), a quarter of the gate
//                logits each, then the hx_moe / x_moe router of token 1
//   warps 2..5   the cx_moe router of token 0 (a quarter of the inputs each; its input and gate
//   warps 6..9   logits come from the previous kernels, so it runs while attention does)
//
// Steps and rounding are those of row_attn_kernel (one/modeling_one.py:390-556,
// one/linear_moe.py:53-90): the routers use the same helpers (warp_gate_factors,
// warp_expert_sums_t, topk_select_fast, warp_combine).
#pragma once

#include "attn_tok.cuh"
#include "common.cuh"
#include "rows.cuh"
#include "topk.cuh"

namespace one {

constexpr int kDecThreads = 384;

struct DecAttnParams {
  int T, H, r, E, k;
  const int* counters;   // counters[0] = position of the step's token
  const float* inv_freq;
  const __nv_bfloat16* proj;  // [T][3 * H * Dh]: lin1 | lin2 | lin3 outputs
  float scale;
  uint32_t scale2;
  int scale_exact;
  const __nv_bfloat16 *wq, *bq, *wk, *bk, *wv, *bv;
  MoeRouter rt[3];       // hx_moe, x_moe (gate_w [r, H*H]), cx_moe (glog precomputed, x = clamp(cx))
  unsigned long long tie;
  DevErr* err;
  int mode;              // kAttnFeature, or kAttnValue (use_flash_attention: o = v for a one-token call)
};

// Shared memory (byte offsets).
struct DecTokLayout {
  int rows, stage, xs, cxs, gl, gq, cv, part, scr, sc, sel, bytes;
};
struct DecLayout {
  int ws, bs, g16, exps, b2, tab, tok0, total;
  DecTokLayout tk;
};
template <int DH>
__host__ __device__ inline DecLayout dec_layout(int H, int r, int E, int D) {
  constexpr int RS = DH + 16;
  DecLayout L;
  const int HH = H * H;
  int off = 0;
  L.ws = attn_take(off, 3 * 16 * RS * 2);
  L.bs = attn_take(off, 3 * 16 * 4);
  L.g16 = attn_take(off, 2 * r * HH * 2);
  L.exps = attn_take(off, 3 * E * 4);
  L.b2 = attn_take(off, E * (2 * HH + D) * 2);
  L.tab = attn_take(off, DH * 2);
  L.tok0 = off;
  int t = 0;
  DecTokLayout& k = L.tk;
  k.rows = attn_take(t, 3 * H * RS * 2);
  k.stage = attn_take(t, HH * 2);
  k.xs = attn_take(t, HH * 4);
  k.cxs = attn_take(t, D * 4);
  k.gl = attn_take(t, 3 * r * 4);
  k.gq = attn_take(t, 4 * r * 4);
  k.cv = attn_take(t, 6 * E * 4);
  k.part = attn_take(t, 4 * kMaxExperts * 8);
  k.scr = attn_take(t, 6 * 32 * 8);
  k.sc = attn_take(t, 3 * E * 4);
  k.sel = attn_take(t, 3 * E * 4);
  k.bytes = t;
  L.total = off + 2 * t;
  return L;
}

template <int DH>
__global__ void __launch_bounds__(kDecThreads, 1) dec_attn_kernel(const DecAttnParams p) {
  extern __shared__ __align__(16) uint8_t smb[];
  using T = __nv_bfloat16;
  const int H = p.H, HD = H * DH, HH = H * H, r = p.r, E = p.E;
  const int D = p.rt[2].in;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, c = lane & 3;
  const DecLayout L = dec_layout<DH>(H, r, E, D);
  __nv_bfloat16* ws = reinterpret_cast<__nv_bfloat16*>(smb + L.ws);
  float* bs = reinterpret_cast<float*>(smb + L.bs);
  T* g16 = reinterpret_cast<T*>(smb + L.g16);
  float* exps = reinterpret_cast<float*>(smb + L.exps);
  T* b2s = reinterpret_cast<T*>(smb + L.b2);
  const int b2off[3] = {0, E * HH, 2 * E * HH};
  const int inr[3] = {HH, HH, D};

  // ---- weights (never written by the preceding kernels): staged before the dependency wait
  stage_head_proj<DH>(ws, bs, H, p.wq, p.bq, p.wk, p.bk, p.wv, p.bv);
  {
    const int ng = r * HH * 2 / 16;
    uint4* gd = reinterpret_cast<uint4*>(g16);
    for (int v = tid; v < 2 * ng; v += blockDim.x)
      gd[v] = reinterpret_cast<const uint4*>(p.rt[v / ng].gate_w)[v % ng];
  }
  for (int i = tid; i < 3 * E; i += blockDim.x)
    exps[i] = fminf(fmaxf(ld<T>(reinterpret_cast<const T*>(p.rt[i / E].experts) + i % E), -10.f), 10.f);
  for (int ri = 0; ri < 3; ++ri) {
    const uint4* src = reinterpret_cast<const uint4*>(p.rt[ri].bias2);
    uint4* dst = reinterpret_cast<uint4*>(b2s + b2off[ri]);
    for (int v = tid; v < E * inr[ri] / 8; v += blockDim.x) dst[v] = src[v];
  }
  __syncthreads();
  if (tid == 0) pdl_launch_dependents();
  pdl_wait();

  const int kk = min(p.k, E);
  __nv_bfloat16* tab = reinterpret_cast<__nv_bfloat16*>(smb + L.tab);
  if (warp >= 10) {
    // cos / sin of the step's position (OneRotaryEmbedding, :159-182), one index per lane
    const int pos = p.counters[0];
    for (int i = tid - 320; i < DH / 2; i += 64) {
      const float f = p.inv_freq[i] * (float)pos;
      tab[i] = __float2bfloat16_rn(cosf(f));
      tab[DH / 2 + i] = __float2bfloat16_rn(sinf(f));
    }
    named_bar(5, 128);
  }
  bool first = true;
  for (int t0 = blockIdx.x * 2; t0 < p.T; t0 += gridDim.x * 2) {
    const int ntok = min(2, p.T - t0);
    if (warp < 2) {
      // ---- attention of token `warp`, then the gate logits of both tokens
      const int k = warp;
      uint8_t* tb = smb + L.tok0 + k * L.tk.bytes;
      __nv_bfloat16* rows = reinterpret_cast<__nv_bfloat16*>(tb + L.tk.rows);
      uint32_t* stage = reinterpret_cast<uint32_t*>(tb + L.tk.stage);
      float* xs = reinterpret_cast<float*>(tb + L.tk.xs);
      if (k < ntok) load_token_rows<DH>(p.proj + (size_t)(t0 + k) * 3 * HD, H, rows);
      if (first) named_bar(5, 128);  // the cos / sin table
      if (k < ntok) {
        uint2 cs[DH / 32], sn[DH / 32];
#pragma unroll
        for (int ls = 0; ls < DH / 32; ++ls) {
          cs[ls] = *reinterpret_cast<const uint2*>(tab + ls * 16 + 4 * c);
          sn[ls] = *reinterpret_cast<const uint2*>(tab + DH / 2 + ls * 16 + 4 * c);
        }
        __syncwarp();
        attn_token_warp<DH>(rows, cs, sn, ws, bs, H, p.scale, p.scale2, p.scale_exact, 0x461c461cu, stage, p.mode);
        __syncwarp();
        for (int w = lane; w < HH / 2; w += 32) {
          const uint32_t u = stage[w];
          reinterpret_cast<float2*>(xs)[w] = make_float2(bf2_lo(u), bf2_hi(u));
        }
      }
    }
    if (warp < 2 || warp >= 10) {
      named_bar(1, 128);  // both tokens' attention outputs
      // gate logits (:56) of both tokens on the CUDA cores: thread u of the four warps takes
      // the gate rows u, u + 128, ... of [hx_moe; x_moe] ([2r][HH]), an fp32 dot product over
      // k in order for each token, rounded to bf16
      const int u = (warp < 2 ? warp : warp - 8) * 32 + lane;
      const float* x0 = reinterpret_cast<const float*>(smb + L.tok0 + L.tk.xs);
      const float* x1 = reinterpret_cast<const float*>(smb + L.tok0 + L.tk.bytes + L.tk.xs);
      for (int jr = u; jr < 2 * r; jr += 128) {
        const T* wrow = g16 + (size_t)jr * HH;
        float a0 = 0.f, a1 = 0.f;
        for (int kq = 0; kq < HH; kq += 8) {
          float w[8];
          load8(wrow + kq, w);
          const float4 p0 = *reinterpret_cast<const float4*>(x0 + kq), p1 = *reinterpret_cast<const float4*>(x0 + kq + 4);
          const float4 q0 = *reinterpret_cast<const float4*>(x1 + kq), q1 = *reinterpret_cast<const float4*>(x1 + kq + 4);
          a0 = fmaf(w[0], p0.x, a0); a0 = fmaf(w[1], p0.y, a0); a0 = fmaf(w[2], p0.z, a0); a0 = fmaf(w[3], p0.w, a0);
          a0 = fmaf(w[4], p1.x, a0); a0 = fmaf(w[5], p1.y, a0); a0 = fmaf(w[6], p1.z, a0); a0 = fmaf(w[7], p1.w, a0);
          a1 = fmaf(w[0], q0.x, a1); a1 = fmaf(w[1], q0.y, a1); a1 = fmaf(w[2], q0.z, a1); a1 = fmaf(w[3], q0.w, a1);
          a1 = fmaf(w[4], q1.x, a1); a1 = fmaf(w[5], q1.y, a1); a1 = fmaf(w[6], q1.z, a1); a1 = fmaf(w[7], q1.w, a1);
        }
        const int ri = jr / r, j = jr % r;
        reinterpret_cast<float*>(smb + L.tok0 + L.tk.gl)[ri * r + j] = rnd<T>(a0);
        if (ntok > 1) reinterpret_cast<float*>(smb + L.tok0 + L.tk.bytes + L.tk.gl)[ri * r + j] = rnd<T>(a1);
      }
      named_bar(2, 128);
    }
    if (warp < 2 || warp >= 10) {
      // ---- hx_moe (ri 0) / x_moe (ri 1) router of token k on clamp(o)
      const int k = warp < 2 ? 0 : 1, ri = warp & 1;
      if (k < ntok) {
        const int t = t0 + k;
        uint8_t* tb = smb + L.tok0 + k * L.tk.bytes;
        const float* xs = reinterpret_cast<const float*>(tb + L.tk.xs);
        float* gl = reinterpret_cast<float*>(tb + L.tk.gl) + ri * r;
        float* cv = reinterpret_cast<float*>(tb + L.tk.cv) + ri * E;
        float* sc = reinterpret_cast<float*>(tb + L.tk.sc) + ri * E;
        int* sel = reinterpret_cast<int*>(tb + L.tk.sel) + ri * E;
        double* scr = reinterpret_cast<double*>(tb + L.tk.scr) + ri * 32;
        warp_gate_factors<T>(gl, r, exps + ri * E, E, cv, scr);
        const T* B2 = b2s + b2off[ri];
        for (int e0 = 0; e0 < E; e0 += 8) {
          const double tot = warp_expert_sums_t<T>(xs, 0, HH, B2, HH, cv, e0, E);
          const int sl = e0 + r2_slot(lane);
          if ((lane & 3) == 0 && sl < E) sc[sl] = rnd<T>(__double2float_rn(tot));
        }
        __syncwarp();
        if (lane == 0) {
          int chosen[kMaxExperts];
          topk_select_fast(sc, E, kk, chosen, p.tie);
          for (int j = 0; j < kk; ++j) {
            sel[j] = chosen[j];
            if (p.rt[ri].idx_out) p.rt[ri].idx_out[(size_t)t * kk + j] = chosen[j];
          }
        }
        __syncwarp();
        warp_combine<T>(xs, 0, HH, B2, HH, cv, sel, kk, reinterpret_cast<T*>(p.rt[ri].comb) + (size_t)t * HH);
      }
    } else {
      // ---- cx_moe router: warps 2..5 token 0, 6..9 token 1, a quarter of the inputs each
      const int k = (warp - 2) >> 2, q = (warp - 2) & 3;
      if (k < ntok) {
        const int t = t0 + k;
        uint8_t* tb = smb + L.tok0 + k * L.tk.bytes;
        float* cxs = reinterpret_cast<float*>(tb + L.tk.cxs);
        float* gq = reinterpret_cast<float*>(tb + L.tk.gq) + q * r;
        float* cv = reinterpret_cast<float*>(tb + L.tk.cv) + (2 + q) * E;
        double* part = reinterpret_cast<double*>(tb + L.tk.part);
        float* sc = reinterpret_cast<float*>(tb + L.tk.sc) + 2 * E;
        int* sel = reinterpret_cast<int*>(tb + L.tk.sel) + 2 * E;
        const int qlen = (((D + 3) / 4) + 7) & ~7;  // quarters on 8-element boundaries
        const int i0 = min(D, q * qlen), i1 = min(D, i0 + qlen);
        const T* X = reinterpret_cast<const T*>(p.rt[2].x) + (size_t)t * p.rt[2].ldx;
        for (int i = i0 + 8 * lane; i < i1; i += 256) {
          float v[8];
          load8(X + i, v);
#pragma unroll
          for (int e = 0; e < 8; ++e) cxs[i + e] = v[e];  // already clamped (clamp(cx) from the GEMM epilogue)
        }
        const T* GL = reinterpret_cast<const T*>(p.rt[2].glog) + (size_t)t * r;
        for (int j = lane; j < r; j += 32) gq[j] = ld<T>(GL + j);
        __syncwarp();
        warp_gate_factors<T>(gq, r, exps + 2 * E, E, cv, reinterpret_cast<double*>(tb + L.tk.scr) + (2 + q) * 32);
        const T* B2 = b2s + b2off[2];
        for (int e0 = 0; e0 < E; e0 += 8) {
          const double tot = warp_expert_sums_t<T>(cxs, i0, i1, B2, D, cv, e0, E);
          const int sl = e0 + r2_slot(lane);
          if ((lane & 3) == 0 && sl < E) part[q * kMaxExperts + sl] = tot;
        }
        named_bar(3 + k, 128);
        if (q == 0) {
          for (int e = lane; e < E; e += 32) {  // the quarters' partials added in quarter order
            double s2 = 0.0;
            for (int qq = 0; qq < 4; ++qq) s2 += part[qq * kMaxExperts + e];
            sc[e] = rnd<T>(__double2float_rn(s2));
          }
          __syncwarp();
          if (lane == 0) {
            int chosen[kMaxExperts];
            topk_select_fast(sc, E, kk, chosen, p.tie);
            for (int j = 0; j < kk; ++j) {
              sel[j] = chosen[j];
              if (p.rt[2].idx_out) p.rt[2].idx_out[(size_t)t * kk + j] = chosen[j];
            }
          }
        }
        named_bar(3 + k, 128);
        warp_combine<T>(cxs, i0, i1, B2, D, cv, sel, kk, reinterpret_cast<T*>(p.rt[2].comb) + (size_t)t * D);
      }
    }
    first = false;
    __syncthreads();
  }
}

}  // namespace one
