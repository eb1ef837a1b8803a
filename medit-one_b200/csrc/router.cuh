// LinearMoE router for bf16 tensors (one/linear_moe.py:53-90) with each token's inputs held
// in registers as packed bf16x2 pairs: lane l owns the input pairs l, l + 32, ... (NP of
// them). Same steps and rounding as moe_router_kernel:
//   x.clamp(-1e4, 1e4)                                   packed min / max against bf16(1e4)
//   gate softmax over r logits (fp32, rounded)           :56
//   c_e = 1 + silu(clamp(mean_j rnd(g_j * experts_e)))   :59-68, exact fp64 sums
//   score_e = sum_i rnd(rnd(x_i * c_e) + bias2[e, i])    :71-80, exact fp64 sums
//   top-k in the reference's selection order             :83-84 (one token per lane)
//   mean of the chosen biased inputs, fp32 in order      :87-90
// Every rounded elementwise step is one packed bf16x2 instruction with round-to-nearest:
// the operands are bf16 values, so one rounding of the exact result equals the
// reference's fp32-then-bf16 rounding. The per-expert fp64 partial sums of a warp are
// reduced with a transposed butterfly (9 double shuffles for 8 experts); the terms are
// bf16 numbers whose fp64 sums do not depend on the order.
#pragma once

#include "common.cuh"
#include "rows.cuh"
#include "topk.cuh"

namespace one {

constexpr int kR2Warps = 8;
constexpr int kR2MaxK = 8;

// Shared memory: bias2 [E][in] bf16 (when it fits), clamped experts [kMaxExperts] fp32,
// per warp the group's expert factors, scores and selections [32][E] each, and (staged) a
// two-token ring of input rows [2][in] and gate-logit rows [2][r] that cp.async fills one
// token ahead of its use.
struct Router2Smem {
  int b2, ex, warp0, per_warp, cf, sc, sel, xs, gs, total, warps;
  bool stage_b2;
};
__host__ __device__ inline Router2Smem router2_smem(int in, int E, int r, bool staged) {
  Router2Smem L;
  const int b2 = E * in * 2;
  L.stage_b2 = b2 <= 48 * 1024;
  L.b2 = 0;
  L.ex = L.stage_b2 ? (b2 + 15) & ~15 : 0;
  L.warp0 = L.ex + kMaxExperts * 4;
  L.cf = 0;
  L.sc = 32 * E * 4;
  L.sel = 2 * 32 * E * 4;
  L.xs = 3 * 32 * E * 4;
  L.gs = L.xs + (staged ? 2 * in * 2 : 0);
  L.per_warp = L.gs + (staged ? 2 * r * 2 : 0);
  const int fit = (200 * 1024 - L.warp0) / L.per_warp;
  L.warps = fit < kR2Warps ? fit : kR2Warps;
  L.total = L.warp0 + (L.warps > 0 ? L.warps : 1) * L.per_warp;
  return L;
}

// NP = input pairs per lane (in <= 64 * NP); r <= 128; k <= kR2MaxK; E <= kMaxExperts.
// staged (in and r multiples of 8, x / glog rows 16-byte aligned): each token's input row and
// gate logits are copied to the warp's ring by cp.async while the previous token computes.
template <int NP>
__global__ void __launch_bounds__(kR2Warps * 32, NP <= 6 ? 3 : 2) moe_router_bf16_kernel(const MoeRouter R, int ntok, int r, int E, int k,
                                                                      int group, unsigned long long tie, int staged) {
  extern __shared__ __align__(16) uint8_t rsm[];
  const int in = R.in, hp = in / 2, lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarp = blockDim.x >> 5;
  const bool stg = NP >= 12 && staged != 0;  // the narrow instantiations carry no staging code
  const Router2Smem L = router2_smem(in, E, r, stg);
  float* exs = reinterpret_cast<float*>(rsm + L.ex);
  uint8_t* wb = rsm + L.warp0 + warp * L.per_warp;
  float* cf = reinterpret_cast<float*>(wb + L.cf);  // [32][E] expert factors of the group
  float* sc = reinterpret_cast<float*>(wb + L.sc);  // [32][E] scores
  int* sel = reinterpret_cast<int*>(wb + L.sel);    // [32][E] chosen experts
  uint8_t* xs = wb + L.xs;                          // staged: [2][in] bf16 input rows
  uint8_t* gs = wb + L.gs;                          // staged: [2][r] bf16 gate logits
  // bias2 and the experts are weights: staged before the dependency wait
  const uint32_t* B2 = reinterpret_cast<const uint32_t*>(R.bias2);
  if (L.stage_b2) {
    uint32_t* b2s = reinterpret_cast<uint32_t*>(rsm + L.b2);
    for (int v = threadIdx.x; v < E * hp; v += blockDim.x) b2s[v] = B2[v];
    B2 = b2s;
  }
  for (int e = threadIdx.x; e < kMaxExperts; e += blockDim.x)
    exs[e] = e < E ? fminf(fmaxf(__bfloat162float(reinterpret_cast<const __nv_bfloat16*>(R.experts)[e]), -10.f), 10.f)
                   : 0.f;
  __syncthreads();
  pdl_wait();
  const int kk = min(k, E);
  const bool pow2k = (kk & (kk - 1)) == 0;
  const float invk = 1.0f / (float)kk;
  const uint32_t cmax = 0x461c461cu, cmin = 0xc61cc61cu;  // +-bf16(1e4) = +-9984
  const int slot = r2_slot(lane);
  const bool two_g = r > 64;
  auto load_x = [&](const uint32_t* X, uint32_t (&xv)[NP]) {
#pragma unroll
    for (int m = 0; m < NP; ++m) {
      const int pi = lane + 32 * m;
      xv[m] = pi < hp ? bf2_min(bf2_max(X[pi], cmin), cmax) : 0u;  // (:53)
    }
  };
  auto x_row = [&](int t) { return reinterpret_cast<const uint32_t*>(R.x) + (size_t)t * (R.ldx / 2); };
  // staged: token u's row (and gate logits) into ring slot u & 1; one commit group per call
  auto stage = [&](int t0, int u, int nt, bool glog) {
    if (u < nt) {
      const uint8_t* src = reinterpret_cast<const uint8_t*>(x_row(t0 + u));
      uint8_t* dst = xs + (u & 1) * in * 2;
      for (int c = lane; c < in / 8; c += 32) cp_async16(dst + c * 16, src + c * 16);
      if (glog) {
        const uint8_t* gsrc = reinterpret_cast<const uint8_t*>(R.glog) + (size_t)(t0 + u) * r * 2;
        if (lane < r / 8) cp_async16(gs + (u & 1) * r * 2 + lane * 16, gsrc + lane * 16);
      }
    }
    cp_async_commit();
  };
  group = max(1, min(32, group));
  for (int t0 = (blockIdx.x * nwarp + warp) * group; t0 < ntok; t0 += gridDim.x * nwarp * group) {
    const int nt = min(group, ntok - t0);
    if (stg) stage(t0, 0, nt, true);
    for (int u = 0; u < nt; ++u) {
      const int t = t0 + u;
      uint32_t xv[NP];
      const __nv_bfloat16* G = reinterpret_cast<const __nv_bfloat16*>(R.glog) + (size_t)t * r;
      if (stg) {
        stage(t0, u + 1, nt, true);
        cp_async_wait<1>();  // token u's copies (this lane's) have landed ...
        __syncwarp();        // ... and every lane's
        load_x(reinterpret_cast<const uint32_t*>(xs + (u & 1) * in * 2), xv);
        G = reinterpret_cast<const __nv_bfloat16*>(gs + (u & 1) * r * 2);
      } else {
        load_x(x_row(t), xv);
      }
      // ---- gate softmax (:56) and expert factors (:59-68)
      float gv[4];
      float mx = -INFINITY;
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        const int j = lane + 32 * m;
        gv[m] = j < r ? __bfloat162float(G[j]) : -INFINITY;
        mx = fmaxf(mx, gv[m]);
      }
      mx = warp_max(mx);
      float sum = 0.f;
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        gv[m] = lane + 32 * m < r ? expf(gv[m] - mx) : 0.f;
        sum += gv[m];
      }
      sum = warp_sum(sum);
      const float inv = 1.0f / sum;
      const uint32_t gp0 = pack_bf16x2(gv[0] * inv, gv[1] * inv), gp1 = pack_bf16x2(gv[2] * inv, gv[3] * inv);
      for (int e0 = 0; e0 < E; e0 += 8) {
        double a[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const uint32_t xe2 = bf2_splat(exs[e0 + e < kMaxExperts ? e0 + e : 0]);
          const uint32_t p0 = bf2_mul(gp0, xe2);
          a[e] = (double)bf2_lo(p0);
          a[e] += (double)bf2_hi(p0);
          if (two_g) {
            const uint32_t p1 = bf2_mul(gp1, xe2);
            a[e] += (double)bf2_lo(p1);
            a[e] += (double)bf2_hi(p1);
          }
        }
        const double tot = warp_transpose_sum8(a);
        if ((lane & 3) == 0 && e0 + slot < E) {
          const float scv = fminf(fmaxf(__bfloat162float(__float2bfloat16_rn((float)tot / (float)r)), -10.f), 10.f);
          cf[u * E + e0 + slot] = __bfloat162float(__float2bfloat16_rn(1.0f + __bfloat162float(__float2bfloat16_rn(silu_f(scv)))));
        }
      }
      __syncwarp();
      // ---- expert scores (:71-80)
      for (int e0 = 0; e0 < E; e0 += 8) {
        uint32_t c2[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) c2[e] = e0 + e < E ? bf2_splat(cf[u * E + e0 + e]) : 0u;
        double a[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) a[e] = 0.0;
#pragma unroll
        for (int m = 0; m < NP; ++m) {
          const int pi = lane + 32 * m;
          if (pi < hp) {
#pragma unroll
            for (int e = 0; e < 8; ++e)
              if (e0 + e < E) {
                const uint32_t rr = bf2_add(bf2_mul(xv[m], c2[e]), B2[(e0 + e) * hp + pi]);
                a[e] += (double)bf2_lo(rr);
                a[e] += (double)bf2_hi(rr);
              }
          }
        }
        const double tot = warp_transpose_sum8(a);
        if ((lane & 3) == 0 && e0 + slot < E) sc[u * E + e0 + slot] = __bfloat162float(__float2bfloat16_rn(__double2float_rn(tot)));
      }
      if (stg) __syncwarp();  // ring slot u & 1 is refilled by the next token's stage
    }
    if (stg) cp_async_wait<0>();
    __syncwarp();
    if (lane < nt) {  // top-k (:83-84), one token per lane
      topk_select_fast(sc + lane * E, E, kk, sel + lane * E, tie);
      if (R.idx_out)
        for (int j = 0; j < kk; ++j) R.idx_out[(size_t)(t0 + lane) * kk + j] = sel[lane * E + j];
    }
    __syncwarp();
    if (stg) stage(t0, 0, nt, false);
    for (int u = 0; u < nt; ++u) {  // mean of the chosen biased inputs (:87-90)
      const int t = t0 + u;
      uint32_t xv[NP];
      if (stg) {
        stage(t0, u + 1, nt, false);
        cp_async_wait<1>();
        __syncwarp();
        load_x(reinterpret_cast<const uint32_t*>(xs + (u & 1) * in * 2), xv);
      } else {
        load_x(x_row(t), xv);
      }
      int se[kR2MaxK];
      uint32_t sc2[kR2MaxK];
#pragma unroll
      for (int j = 0; j < kR2MaxK; ++j) {
        se[j] = j < kk ? sel[u * E + j] : 0;
        sc2[j] = j < kk ? bf2_splat(cf[u * E + se[j]]) : 0u;
      }
      uint32_t* out = reinterpret_cast<uint32_t*>(R.comb) + (size_t)t * hp;
#pragma unroll
      for (int m = 0; m < NP; ++m) {
        const int pi = lane + 32 * m;
        if (pi < hp) {
          float s0 = 0.f, s1 = 0.f;
#pragma unroll
          for (int j = 0; j < kR2MaxK; ++j)
            if (j < kk) {
              const uint32_t rr = bf2_add(bf2_mul(xv[m], sc2[j]), B2[se[j] * hp + pi]);
              s0 += bf2_lo(rr);
              s1 += bf2_hi(rr);
            }
          out[pi] = pow2k ? pack_bf16x2(s0 * invk, s1 * invk) : pack_bf16x2(s0 / (float)kk, s1 / (float)kk);
        }
      }
      if (stg) __syncwarp();  // ring slot u & 1 is refilled by the next token's stage
    }
    if (stg) cp_async_wait<0>();
    __syncwarp();
  }
}

}  // namespace one
