// Prompt-ingestion feature attention, one warp per token (bf16 models, H <= 16 heads,
// even H, head_dim 32 or 64).
//
// The decode kernel (row_attn_kernel) is shaped for the latency of 256 tokens; a prompt
// call has 10^5..10^6 tokens, so here every warp takes whole tokens with no CTA-wide
// barrier after the weights are staged, and the routers run afterwards as separate
// launches (gate GEMM on the tensor cores, moe_router_kernel).
//
// Per token (one/modeling_one.py:390-556): q = single_x * scale, RoPE (rotate_half) on q and
// on the key, the three head projections lin_q / lin_k / lin_v (Dh -> H) as one m16n8k16
// mma.sync chain with the heads as the M rows, bias, logits q * k, softmax over the H
// outputs of each head (fp32, rounded), o = w * v. Every elementwise step that the
// reference rounds to bf16 is computed on packed bf16x2 operands with an explicit
// round-to-nearest instruction: for bf16 inputs the fp32 product of two values is exact
// and an fp32 sum that is inexact lies far from any bf16 rounding boundary, so one
// rounding of the exact result equals the reference's fp32-then-bf16 rounding.
#pragma once

#include "common.cuh"
#include "rows.cuh"

namespace one {

constexpr int kTokWarps = 8;

// What attn_token_warp produces for a token (one/modeling_one.py:408-547):
//   kAttnFeature  the feature attention o = softmax(q * k) * v per head (use_flash_attention off)
//   kAttnValue    o = v: the flash-attention path over a call of one token, whose causal
//                 attention sees that token only, so the softmax weight is exactly 1
//   kAttnQKV      the projected q | k | v rows themselves ([3][H][H] bf16, bias added), for the
//                 flash-attention path's causal attention across the call's tokens
enum : int { kAttnFeature = 0, kAttnValue = 1, kAttnQKV = 2 };

struct AttnTokParams {
  int T, H, seq_len;
  const __nv_bfloat16* rope;  // [seq_len][Dh]: cos(f_i) for i < Dh/2, then sin(f_i); f_i = inv_freq_i * (pos0 + s)
  const __nv_bfloat16* proj;  // [T][3 * H * Dh]: lin1 | lin2 | lin3 outputs (bias added)
  float scale;                // attention scale 1/sqrt(Dh)
  uint32_t scale2;            // the scale as bf16x2, when scale_exact (a bf16 value)
  int scale_exact;
  const __nv_bfloat16 *wq, *bq, *wk, *bk, *wv, *bv;  // lin_q / lin_k / lin_v [H, Dh], [H]
  __nv_bfloat16* out;         // [T][H * H] (mode kAttnQKV: [T][out_ld] rows of q | k | v, 3 H * H each)
  uint32_t clamp2;            // bf16x2 bound of the LinearMoE input clamp (0: store o unclamped)
  int mode;                   // kAttnFeature or kAttnQKV
  int out_ld;                 // elements per output row
};

// Per-position tables of one prompt call, shared by all layers: the RoPE cos / sin
// (OneRotaryEmbedding, one/modeling_one.py:159-182: the fp32 angle inv_freq_i * pos, cos / sin
// rounded to bf16) and the reciprocal of each prefix-mean divisor (for div_rn_recip).
struct PromptTabParams {
  const int* counters;  // counters[0] = position of the first prompt token
  const float* inv_freq;
  int seq_len, half;    // half = 0: no RoPE table
  __nv_bfloat16* tab;   // [seq_len][2 * half]
  const float* div;     // [seq_len] prefix-mean divisors
  float2* dr;           // [seq_len] (div, RN(1 / div))
};

__global__ void prompt_table_kernel(const PromptTabParams p) {
  pdl_wait();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < p.seq_len) p.dr[i] = make_float2(p.div[i], 1.0f / p.div[i]);
  if (i >= p.seq_len * p.half) return;
  const int s = i / p.half, j = i % p.half;
  const float f = p.inv_freq[j] * (float)(p.counters[0] + s);
  p.tab[(size_t)s * 2 * p.half + j] = __float2bfloat16_rn(cosf(f));
  p.tab[(size_t)s * 2 * p.half + p.half + j] = __float2bfloat16_rn(sinf(f));
}

// Shared memory (bytes): lin_q / lin_k / lin_v as [3][16][RS] bf16 (rows >= H zero), biases
// [3][16] fp32, then per warp two buffers of a token's q | k | v rows [3H][RS] bf16 (the next
// token's rows are copied in by cp.async while the current token computes) and the output
// row [H*H] bf16. RS = Dh + 16: a row stride of 8 (mod 32) words makes the warp's 8-byte
// fragment loads (8 rows x 4 column groups) conflict-free.
template <int DH>
struct AttnTokSmem {
  static constexpr int RS = DH + 16;
  static constexpr int W = 0;
  static constexpr int BIAS = 3 * 16 * RS * 2;
  static constexpr int WARP0 = BIAS + 3 * 16 * 4;
  __host__ __device__ static int rows_bytes(int H) { return 3 * H * RS * 2; }
  __host__ __device__ static int per_warp(int H) { return (2 * rows_bytes(H) + 3 * H * H * 2 + 15) & ~15; }
  __host__ __device__ static int total(int H) { return WARP0 + kTokWarps * per_warp(H); }
};

// Stage lin_q / lin_k / lin_v ([3][16][RS] bf16, rows >= H zero) and their biases ([3][16]
// fp32) into shared memory, all threads of the CTA.
template <int DH>
ONE_DEVINL void stage_head_proj(__nv_bfloat16* ws, float* bs, int H, const __nv_bfloat16* wq, const __nv_bfloat16* bq,
                                const __nv_bfloat16* wk, const __nv_bfloat16* bk, const __nv_bfloat16* wv,
                                const __nv_bfloat16* bv) {
  constexpr int RS = DH + 16, NCH = DH / 8;
  for (int v = threadIdx.x; v < 3 * 16 * NCH; v += blockDim.x) {
    const int row = v / NCH, ch = v % NCH, pj = row / 16, n = row % 16;
    uint4 val = make_uint4(0u, 0u, 0u, 0u);
    if (n < H) {
      const __nv_bfloat16* W = pj == 0 ? wq : pj == 1 ? wk : wv;
      val = *reinterpret_cast<const uint4*>(W + (size_t)n * DH + ch * 8);
    }
    *reinterpret_cast<uint4*>(ws + row * RS + ch * 8) = val;
  }
  for (int i = threadIdx.x; i < 3 * 16; i += blockDim.x) {
    const int pj = i / 16, n = i % 16;
    const __nv_bfloat16* B = pj == 0 ? bq : pj == 1 ? bk : bv;
    bs[i] = n < H ? __bfloat162float(B[n]) : 0.f;
  }
}

// One warp copies a token's q | k | v row ([3 * H * DH] bf16) into rows [3H][RS].
template <int DH>
ONE_DEVINL void load_token_rows(const __nv_bfloat16* src_row, int H, __nv_bfloat16* rows) {
  constexpr int RS = DH + 16, NCH = DH / 8, kMaxLd = (3 * 16 * NCH + 31) / 32;
  const int lane = threadIdx.x & 31, nch = 3 * H * NCH;
  const uint4* src = reinterpret_cast<const uint4*>(src_row);
  uint4 v[kMaxLd];
#pragma unroll
  for (int m = 0; m < kMaxLd; ++m) {
    const int j = lane + 32 * m;
    if (j < nch) v[m] = src[j];
  }
#pragma unroll
  for (int m = 0; m < kMaxLd; ++m) {
    const int j = lane + 32 * m;
    if (j < nch) *reinterpret_cast<uint4*>(rows + (j / NCH) * RS + (j % NCH) * 8) = v[m];
  }
}

// Fragment layout of the projections: m16n8k16 with rows = heads g and g + 8, columns =
// outputs. Within each 16-wide k slice, lane (g, c) supplies the logical k = 4c..4c+3 (one
// 8-byte load) as the hardware's k = {2c, 2c+1, 2c+8, 2c+9}; A and B use the same
// assignment, so every product pairs the same (k) elements. cs / sn: the lane's cos / sin
// pairs of indices 16 ls + 4c + {0, 1} (.x) and {2, 3} (.y), ls < DH / 32.
//
// One token by one warp: rows = the token's q | k | v ([3H][RS] bf16), ws / bs the staged
// projections; writes the output row (clamped to +-clamp2 when clamp2 != 0) as bf16 pairs
// into stage[H*H/2], or with mode kAttnQKV the unclamped q | k | v rows into stage[3*H*H/2].
template <int DH>
ONE_DEVINL void attn_token_warp(const __nv_bfloat16* rows, const uint2 (&cs)[DH / 32], const uint2 (&sn)[DH / 32],
                                const __nv_bfloat16* ws, const float* bs, int H, float scale, uint32_t scale2,
                                int scale_exact, uint32_t clamp2, uint32_t* stage, int mode = kAttnFeature) {
  constexpr int RS = DH + 16, NS = DH / 16;
  const int lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
  const bool two_nt = H > 8;
  const uint32_t negc = clamp2 ^ 0x80008000u;
  float acc[3][2][4];
#pragma unroll
  for (int pj = 0; pj < 3; ++pj)
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int q = 0; q < 4; ++q) acc[pj][nt][q] = 0.f;
#pragma unroll
  for (int pj = 0; pj < 3; ++pj) {
    uint32_t a[NS][4];
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
      const int h = g + 8 * rr;
      const bool ok = h < H;
      const __nv_bfloat16* rw = rows + (pj * H + (ok ? h : 0)) * RS + 4 * c;
#pragma unroll
      for (int ls = 0; ls < NS / 2; ++ls) {
        uint2 lo = make_uint2(0u, 0u), hi = make_uint2(0u, 0u);
        if (ok) {
          lo = *reinterpret_cast<const uint2*>(rw + ls * 16);
          hi = *reinterpret_cast<const uint2*>(rw + (ls + NS / 2) * 16);
        }
        if (pj < 2) {
          if (pj == 0) {  // single_x * scale (:405)
            if (scale_exact) {
              lo = make_uint2(bf2_mul(lo.x, scale2), bf2_mul(lo.y, scale2));
              hi = make_uint2(bf2_mul(hi.x, scale2), bf2_mul(hi.y, scale2));
            } else {
              lo = make_uint2(pack_bf16x2(bf2_lo(lo.x) * scale, bf2_hi(lo.x) * scale),
                              pack_bf16x2(bf2_lo(lo.y) * scale, bf2_hi(lo.y) * scale));
              hi = make_uint2(pack_bf16x2(bf2_lo(hi.x) * scale, bf2_hi(hi.x) * scale),
                              pack_bf16x2(bf2_lo(hi.y) * scale, bf2_hi(hi.y) * scale));
            }
          }
          // x * cos + rotate_half(x) * sin: out[d] = x[d] cos - x[d + half] sin,
          // out[d + half] = x[d + half] cos + x[d] sin (cos / sin of index d)
          const uint2 rl = make_uint2(bf2_sub(bf2_mul(lo.x, cs[ls].x), bf2_mul(hi.x, sn[ls].x)),
                                      bf2_sub(bf2_mul(lo.y, cs[ls].y), bf2_mul(hi.y, sn[ls].y)));
          const uint2 rh = make_uint2(bf2_add(bf2_mul(hi.x, cs[ls].x), bf2_mul(lo.x, sn[ls].x)),
                                      bf2_add(bf2_mul(hi.y, cs[ls].y), bf2_mul(lo.y, sn[ls].y)));
          lo = rl;
          hi = rh;
        }
        a[ls][rr] = lo.x;
        a[ls][rr + 2] = lo.y;
        a[ls + NS / 2][rr] = hi.x;
        a[ls + NS / 2][rr + 2] = hi.y;
      }
    }
    const __nv_bfloat16* wrow = ws + pj * 16 * RS + 4 * c;
#pragma unroll
    for (int ks = 0; ks < NS; ++ks)
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
        if (nt == 0 || two_nt) {
          const uint2 b = *reinterpret_cast<const uint2*>(wrow + (nt * 8 + g) * RS + ks * 16);
          mma_16816_bf16(acc[pj][nt], a[ks], b.x, b.y);
        }
  }

  // lane (g, c): heads h = g + 8 rr, outputs j = 8 nt + 2c + {0, 1}
#pragma unroll
  for (int rr = 0; rr < 2; ++rr) {
    const int h = g + 8 * rr;
    uint32_t lg[2], vv[2];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      const int j = nt * 8 + 2 * c;
      const uint32_t q2 = pack_bf16x2(acc[0][nt][2 * rr] + bs[j], acc[0][nt][2 * rr + 1] + bs[j + 1]);
      const uint32_t k2 = pack_bf16x2(acc[1][nt][2 * rr] + bs[16 + j], acc[1][nt][2 * rr + 1] + bs[16 + j + 1]);
      vv[nt] = pack_bf16x2(acc[2][nt][2 * rr] + bs[32 + j], acc[2][nt][2 * rr + 1] + bs[32 + j + 1]);
      const uint32_t m = (j < H ? 0u : 0xffffu) | (j + 1 < H ? 0u : 0xffff0000u);
      lg[nt] = (bf2_mul(q2, k2) & ~m) | (0xff80ff80u & m);  // masked outputs: -inf
      if (mode != kAttnFeature && h < H && j < H) {
        if (mode == kAttnQKV) {
          stage[(h * H + j) >> 1] = q2;
          stage[(H * H + h * H + j) >> 1] = k2;
          stage[(2 * H * H + h * H + j) >> 1] = vv[nt];
        } else {
          uint32_t o2 = vv[nt];
          if (clamp2) o2 = bf2_min(bf2_max(o2, negc), clamp2);  // LinearMoE clamp (one/linear_moe.py:53)
          stage[(h * H + j) >> 1] = o2;
        }
      }
    }
    if (mode != kAttnFeature) continue;  // warp-uniform
    uint32_t m2 = bf2_max(lg[0], lg[1]);
    float mx = fmaxf(bf2_lo(m2), bf2_hi(m2));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    const uint32_t mx2 = pack_bf16x2(mx, mx);
    uint32_t d1[2];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) d1[nt] = bf2_sub(lg[nt], mx2);
    m2 = bf2_max(d1[0], d1[1]);
    float mm = fmaxf(bf2_lo(m2), bf2_hi(m2));
    mm = fmaxf(mm, __shfl_xor_sync(0xffffffffu, mm, 1));
    mm = fmaxf(mm, __shfl_xor_sync(0xffffffffu, mm, 2));
    float ex[4], sum = 0.f;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int nt = q >> 1, j = nt * 8 + 2 * c + (q & 1);
      const float d = (q & 1) ? bf2_hi(d1[nt]) : bf2_lo(d1[nt]);
      ex[q] = j < H ? expf(d - mm) : 0.f;
      sum += ex[q];
    }
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    sum += __shfl_xor_sync(0xffffffffu, sum, 2);
    const float inv = 1.0f / sum;
    if (h < H) {
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        const int j = nt * 8 + 2 * c;
        if (j < H) {
          float w0 = ex[2 * nt] * inv, w1 = ex[2 * nt + 1] * inv;
          if (isnan(w0)) w0 = 1.0f / (float)H;
          if (isnan(w1)) w1 = 1.0f / (float)H;
          uint32_t o2 = bf2_mul(pack_bf16x2(w0, w1), vv[nt]);
          if (clamp2) o2 = bf2_min(bf2_max(o2, negc), clamp2);  // LinearMoE clamp (one/linear_moe.py:53)
          stage[(h * H + j) >> 1] = o2;
        }
      }
    }
  }
}

template <int DH>
__global__ void __launch_bounds__(kTokWarps * 32, 2) attn_tok_kernel(const AttnTokParams p) {
  using S = AttnTokSmem<DH>;
  constexpr int RS = S::RS, HALF = DH / 2;
  extern __shared__ __align__(16) uint8_t smb[];
  const int H = p.H, HD = H * DH, HH = H * H;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, c = lane & 3;
  __nv_bfloat16* ws = reinterpret_cast<__nv_bfloat16*>(smb + S::W);
  float* bs = reinterpret_cast<float*>(smb + S::BIAS);
  // weights (never written by the preceding kernels): staged before the dependency wait
  stage_head_proj<DH>(ws, bs, H, p.wq, p.bq, p.wk, p.bk, p.wv, p.bv);
  __syncthreads();
  pdl_wait();

  uint8_t* wb = smb + S::WARP0 + warp * S::per_warp(H);
  uint32_t* stage = reinterpret_cast<uint32_t*>(wb + 2 * S::rows_bytes(H));
  // token t's q | k | v row into buffer b, 16-byte chunks; one commit group per call
  auto issue = [&](int t, int b) {
    if (t < p.T) {
      constexpr int NCH = DH / 8;
      const uint8_t* src = reinterpret_cast<const uint8_t*>(p.proj + (size_t)t * 3 * HD);
      uint8_t* dst = wb + b * S::rows_bytes(H);
      for (int j = lane; j < 3 * H * NCH; j += 32) cp_async16(dst + ((j / NCH) * RS + (j % NCH) * 8) * 2, src + j * 16);
    }
    cp_async_commit();
  };
  const int stride = gridDim.x * kTokWarps;
  int it = 0;
  issue(blockIdx.x * kTokWarps + warp, 0);
  for (int t = blockIdx.x * kTokWarps + warp; t < p.T; t += stride, ++it) {
    issue(t + stride, (it + 1) & 1);
    cp_async_wait<1>();  // this lane's copies of token t have landed ...
    __syncwarp();        // ... and every lane's
    const __nv_bfloat16* rows = reinterpret_cast<const __nv_bfloat16*>(wb + (it & 1) * S::rows_bytes(H));
    const __nv_bfloat16* tab = p.rope + (size_t)(t % p.seq_len) * DH;
    uint2 cs[DH / 32], sn[DH / 32];
#pragma unroll
    for (int ls = 0; ls < DH / 32; ++ls) {
      cs[ls] = *reinterpret_cast<const uint2*>(tab + ls * 16 + 4 * c);
      sn[ls] = *reinterpret_cast<const uint2*>(tab + HALF + ls * 16 + 4 * c);
    }
    __syncwarp();
    attn_token_warp<DH>(rows, cs, sn, ws, bs, H, p.scale, p.scale2, p.scale_exact, p.clamp2, stage, p.mode);
    __syncwarp();
    uint32_t* dst = reinterpret_cast<uint32_t*>(p.out + (size_t)t * p.out_ld);
    const int nw = (p.mode == kAttnQKV ? 3 * HH : HH) / 2;
    for (int w = lane; w < nw; w += 32) dst[w] = stage[w];
    __syncwarp();  // buffer it & 1 is refilled by the next iteration's issue
  }
  cp_async_wait<0>();
}

}  // namespace one
