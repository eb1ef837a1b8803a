// Causal softmax attention across a prompt's tokens, one head of H features at a time: the
// use_flash_attention path of One.forward (one/modeling_one.py:408-421), whose
// TurboFlashAttention(causal=True) is turbo_flash_attention's exact attention
// (one/turbo_ops.py:115-143) with the default scale 1/sqrt(H):
//
//   q' = bf16(q * scale),  s[t, j] = bf16(q'[t] . k[j])  (fp32 sum, one rounding),
//   o[t] = sum_{j <= t} softmax_j(s[t, :]) v[j],  rounded to bf16 once,
//
// per sequence b and head n, over the positions of one prompt call. q, k, v are the per-head
// projections lin_q / lin_k / lin_v of the rotated single_x / key and of value (H outputs
// each), written by attn_tok_kernel in mode kAttnQKV as row t = [q | k | v] ([3][H][H] bf16,
// row stride ld), token t = b * seq_len + position. The output row o[t] ([H][H] bf16) gets the
// LinearMoE input clamp when the layer's MoEs are routed (one/linear_moe.py:53).
//
// One thread per query position, kSeqQ per CTA; keys in tiles of kSeqK staged in shared memory
// as fp32; the softmax is the online form in fp32 (running max and sum; the reference rounds
// each normalised weight to bf16 before the weighted sum, here the weights stay fp32, which
// differs from it by well under one bf16 ulp of the output). Head dims up to kSeqMaxH.
#pragma once

#include "common.cuh"

namespace one {

constexpr int kSeqQ = 128;
constexpr int kSeqK = 64;
constexpr int kSeqMaxH = 16;
constexpr int kSeqGroup = 8;  // keys scored before one online-softmax rescale

struct SeqAttnParams {
  const __nv_bfloat16* qkv;  // row t: q [0, H*H), k [H*H, 2*H*H), v [2*H*H, 3*H*H)
  int ld;                    // elements per qkv row
  __nv_bfloat16* out;        // [T][H*H]
  int seq_len, H;
  float scale;               // 1/sqrt(H)
  float clamp;               // > 0: clamp the output to +-clamp
};

__global__ void __launch_bounds__(kSeqQ) seq_attn_kernel(const SeqAttnParams p) {
  __shared__ float ks[kSeqK][kSeqMaxH + 1], vs[kSeqK][kSeqMaxH + 1];
  pdl_wait();
  const int b = blockIdx.z, n = blockIdx.y, q0 = blockIdx.x * kSeqQ;
  const int H = p.H, HH = H * H;
  const int s = q0 + threadIdx.x;
  const bool valid = s < p.seq_len;
  const size_t base = (size_t)b * p.seq_len;
  float q[kSeqMaxH];
#pragma unroll
  for (int d = 0; d < kSeqMaxH; ++d) {
    q[d] = 0.f;
    if (valid && d < H)
      q[d] = rnd<__nv_bfloat16>(__bfloat162float(p.qkv[(base + s) * p.ld + n * H + d]) * p.scale);
  }
  float m = -INFINITY, l = 0.f, acc[kSeqMaxH];
#pragma unroll
  for (int d = 0; d < kSeqMaxH; ++d) acc[d] = 0.f;
  const int kend = min(p.seq_len, q0 + kSeqQ);  // keys any query of this CTA sees
  for (int k0 = 0; k0 < kend; k0 += kSeqK) {
    __syncthreads();
    for (int i = threadIdx.x; i < kSeqK * H; i += blockDim.x) {
      const int kj = i / H, d = i % H, key = k0 + kj;
      float kv = 0.f, vv = 0.f;
      if (key < p.seq_len) {
        const __nv_bfloat16* row = p.qkv + (base + key) * p.ld + n * H + d;
        kv = __bfloat162float(row[HH]);
        vv = __bfloat162float(row[2 * HH]);
      }
      ks[kj][d] = kv;
      vs[kj][d] = vv;
    }
    __syncthreads();
    if (!valid) continue;
    const int jn = min(kSeqK, s - k0 + 1);  // causal: keys k0 .. s of this tile
    for (int j0 = 0; j0 < jn; j0 += kSeqGroup) {
      float sc[kSeqGroup];
      float gm = -INFINITY;
#pragma unroll
      for (int u = 0; u < kSeqGroup; ++u) {
        const int kj = j0 + u;
        float a = 0.f;
#pragma unroll
        for (int d = 0; d < kSeqMaxH; ++d)
          if (d < H) a = fmaf(q[d], ks[kj < kSeqK ? kj : 0][d], a);
        sc[u] = kj < jn ? rnd<__nv_bfloat16>(a) : -INFINITY;
        gm = fmaxf(gm, sc[u]);
      }
      if (gm > m) {
        const float f = m == -INFINITY ? 0.f : expf(m - gm);
        l *= f;
#pragma unroll
        for (int d = 0; d < kSeqMaxH; ++d) acc[d] *= f;
        m = gm;
      }
#pragma unroll
      for (int u = 0; u < kSeqGroup; ++u) {
        const int kj = j0 + u;
        if (kj >= jn) break;
        const float e = expf(sc[u] - m);
        l += e;
#pragma unroll
        for (int d = 0; d < kSeqMaxH; ++d)
          if (d < H) acc[d] = fmaf(e, vs[kj][d], acc[d]);
      }
    }
  }
  if (!valid) return;
  __nv_bfloat16* o = p.out + (base + s) * HH + n * H;
  const float inv = 1.0f / l;
#pragma unroll
  for (int d = 0; d < kSeqMaxH; ++d) {
    if (d >= H) break;
    float y = rnd<__nv_bfloat16>(acc[d] * inv);
    if (p.clamp > 0.f) y = fminf(fmaxf(y, -p.clamp), p.clamp);
    o[d] = __float2bfloat16_rn(y);
  }
}

}  // namespace one
