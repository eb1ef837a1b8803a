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
// One warp per 16 query positions, four warps per CTA: the scores and the weighted sum run on the
// tensor cores as m16n8k16 bf16 MMAs with the head dim (H <= 16) zero-padded to K = 16:
//   S (16 queries x 16 keys) = Q' K^T    two MMAs (keys 0-7, 8-15)
//   O (16 queries x 16 dims) += P V      two MMAs (dims 0-7, 8-15), P taken straight from S's
//                                        accumulator registers as the A operand
// Keys and values are staged 64 at a time in shared memory (values transposed, key-contiguous).
// The softmax is the online form in fp32 on the bf16-rounded scores (running max and sum per
// query row); P enters the MMAs as a bf16 high part plus the bf16 rounding of its remainder
// (~16 significant bits; the reference rounds each normalised weight to bf16 before its weighted
// sum, which differs from this by well under one bf16 ulp of the output).
#pragma once

#include "common.cuh"
#include "rows.cuh"

namespace one {

constexpr int kSeqQ = 64;     // query positions per CTA (16 per warp)
constexpr int kSeqThreads = 128;
constexpr int kSeqK = 64;     // keys per staged tile
constexpr int kSeqMaxH = 16;  // head dims (zero-padded to the MMA's K = 16)

struct SeqAttnParams {
  const __nv_bfloat16* qkv;  // row t: q [0, H*H), k [H*H, 2*H*H), v [2*H*H, 3*H*H)
  int ld;                    // elements per qkv row
  __nv_bfloat16* out;        // [T][H*H]
  int seq_len, H;
  float scale;               // 1/sqrt(H)
  float clamp;               // > 0: clamp the output to +-clamp
};

__global__ void __launch_bounds__(kSeqThreads) seq_attn_kernel(const SeqAttnParams p) {
  __shared__ __align__(16) __nv_bfloat16 ks[kSeqK][kSeqMaxH + 8];  // keys [key][dim]
  __shared__ __align__(16) __nv_bfloat16 vt[kSeqMaxH][kSeqK + 8];  // values transposed [dim][key]
  pdl_wait();
  using T = __nv_bfloat16;
  const int b = blockIdx.z, n = blockIdx.y, q0 = blockIdx.x * kSeqQ;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
  const int H = p.H, HH = H * H;
  const size_t base = (size_t)b * p.seq_len;
  const int qw = q0 + warp * 16;  // this warp's first query position
  // Q' = bf16(q * scale) as the A fragment: rows qw + g (+8), dims 2c, 2c + 1 (+8)
  auto qv = [&](int row, int d) -> float {
    if (row >= p.seq_len || d >= H) return 0.f;
    return rnd<T>(__bfloat162float(p.qkv[(base + row) * p.ld + n * H + d]) * p.scale);
  };
  uint32_t qa[4];
  qa[0] = pack_bf16x2(qv(qw + g, 2 * c), qv(qw + g, 2 * c + 1));
  qa[1] = pack_bf16x2(qv(qw + g + 8, 2 * c), qv(qw + g + 8, 2 * c + 1));
  qa[2] = pack_bf16x2(qv(qw + g, 2 * c + 8), qv(qw + g, 2 * c + 9));
  qa[3] = pack_bf16x2(qv(qw + g + 8, 2 * c + 8), qv(qw + g + 8, 2 * c + 9));
  float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};  // rows g, g + 8
  float o[2][4];                                              // dims 0-7, 8-15
#pragma unroll
  for (int dt = 0; dt < 2; ++dt)
#pragma unroll
    for (int e = 0; e < 4; ++e) o[dt][e] = 0.f;
  const int kend = min(p.seq_len, q0 + kSeqQ);  // keys any query of this CTA sees
  const int kw = min(kend, qw + 16);             // keys this warp's queries see
  for (int k0 = 0; k0 < kend; k0 += kSeqK) {
    __syncthreads();
    for (int i = threadIdx.x; i < kSeqK * kSeqMaxH; i += blockDim.x) {
      const int kj = i / kSeqMaxH, d = i % kSeqMaxH, key = k0 + kj;
      T kv = __float2bfloat16_rn(0.f), vv = kv;
      if (key < p.seq_len && d < H) {
        const T* row = p.qkv + (base + key) * p.ld + n * H + d;
        kv = row[HH];
        vv = row[2 * HH];
      }
      ks[kj][d] = kv;
      vt[d][kj] = vv;
    }
    __syncthreads();
    const int jend = min(k0 + kSeqK, kw);
    for (int j0 = k0; j0 < jend; j0 += 16) {
      float sc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        const T* kr = &ks[j0 - k0 + nt * 8 + g][0];
        mma_16816_bf16(sc[nt], qa, *reinterpret_cast<const uint32_t*>(kr + 2 * c),
                       *reinterpret_cast<const uint32_t*>(kr + 2 * c + 8));
      }
      // scores as the reference's bf16 matmul rounds them; causal mask and the prompt's end
      float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int key = j0 + nt * 8 + 2 * c + (e & 1), row = qw + g + 8 * (e >> 1);
          sc[nt][e] = (key <= row && key < p.seq_len) ? rnd<T>(sc[nt][e]) : -INFINITY;
          mx[e >> 1] = fmaxf(mx[e >> 1], sc[nt][e]);
        }
      float f[2];
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
        mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
        const float mn = fmaxf(m[r], mx[r]);
        f[r] = mn == -INFINITY ? 1.f : expf(m[r] - mn);
        m[r] = mn;
        l[r] *= f[r];
      }
#pragma unroll
      for (int dt = 0; dt < 2; ++dt) {
        o[dt][0] *= f[0]; o[dt][1] *= f[0];
        o[dt][2] *= f[1]; o[dt][3] *= f[1];
      }
      float pe[2][4];
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float mr = m[e >> 1];
          pe[nt][e] = sc[nt][e] == -INFINITY ? 0.f : expf(sc[nt][e] - mr);
          l[e >> 1] += pe[nt][e];
        }
      // P (16 queries x 16 keys) from the score registers as the A operand, split into a bf16
      // high part and the bf16 rounding of the remainder (two MMAs each), so the weights enter the
      // sum with ~16 significant bits instead of 8
      uint32_t ph[4], pl[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int nt = i >> 1, e0 = (i & 1) * 2;
        ph[i] = pack_bf16x2(pe[nt][e0], pe[nt][e0 + 1]);
        pl[i] = pack_bf16x2(pe[nt][e0] - bf2_lo(ph[i]), pe[nt][e0 + 1] - bf2_hi(ph[i]));
      }
#pragma unroll
      for (int dt = 0; dt < 2; ++dt) {
        const T* vr = &vt[dt * 8 + g][j0 - k0];
        const uint32_t v0 = *reinterpret_cast<const uint32_t*>(vr + 2 * c);
        const uint32_t v1 = *reinterpret_cast<const uint32_t*>(vr + 2 * c + 8);
        mma_16816_bf16(o[dt], ph, v0, v1);
        mma_16816_bf16(o[dt], pl, v0, v1);
      }
    }
  }
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    l[r] += __shfl_xor_sync(0xffffffffu, l[r], 1);
    l[r] += __shfl_xor_sync(0xffffffffu, l[r], 2);
  }
#pragma unroll
  for (int dt = 0; dt < 2; ++dt)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int row = qw + g + 8 * (e >> 1), d = dt * 8 + 2 * c + (e & 1);
      if (row >= p.seq_len || d >= H) continue;
      float y = rnd<T>(o[dt][e] / l[e >> 1]);
      if (p.clamp > 0.f) y = fminf(fmaxf(y, -p.clamp), p.clamp);
      p.out[(base + row) * HH + n * H + d] = __float2bfloat16_rn(y);
    }
}

}  // namespace one
