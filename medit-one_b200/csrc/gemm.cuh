// Weight-stationary GEMMs for the decode / prefill path:
//     Y[t, n] = epilogue( sum_k X[t, k] * W[n, k] )
// W is an nn.Linear weight [N_out, K] (row-major, K contiguous), X the activations
// [T, K]. On the tensor-core path the weight tile is the UMMA "A" operand (M = 128
// rows) and a tile of BN tokens is "B" (N = BN), so one CTA streams a 128-row weight
// slice once and reuses it for BN tokens; both operands arrive by TMA with 128-byte
// swizzle and the fp32 accumulator lives in TMEM. Several independent problems (e.g.
// lin1/lin2/lin3 of one layer, which read different inputs) share one launch.
//
// Epilogues restate the reference's rounding points for the op that follows each
// GEMM (one/modeling_one.py:343-391, 559-573; one/linear_moe.py:93).
#pragma once

#include "common.cuh"

namespace one {

enum EpiKind : int {
  EPI_STORE = 0,    // out = rnd(acc + bias)                                  (nn.Linear)
  EPI_HXPRE = 1,    // out = rnd(aux + clamp(rnd(acc + bias), +-100))         (hx + hx_moe, :559,563)
  EPI_XMOE = 2,     // out = rnd(aux * clamp(rnd(acc + bias), +-100))         (mean * x_moe, :560,568)
  EPI_CX = 3,       // out = rnd(acc + bias); out2 = clamp(out, +-1e4)        (cx_moe, then LinearMoE clamp)
  EPI_GELU_UP = 4,  // rows interleaved (gate j, up j): out[j] = rnd(rnd(gelu(g)) * u)  (OneMLP, :205-206)
  EPI_PARTIAL = 5,  // fp32 split-K partial: ws[split][t][n] = acc
  EPI_ARGMAX = 6,   // logits v = rnd(acc): per-token (max v, lowest n) by 64-bit atomicMax
  EPI_RESID = 7,    // out = rnd(aux + rnd(acc + bias)), bf16, persistent kernel only: the MLP
                    // residual out0 + down_proj(...) (:571) of an unsplit down_proj, in place
};

constexpr int kMaxProblems = 4;

struct GemmProblem {
  int kind;
  int Nw;            // weight rows
  int K;
  int T;             // tokens
  int m_tiles, n_tiles, splits, kb_per_split;
  int m_fast;        // tile order: 1 = weight tile fastest (many token tiles), 0 = token tile fastest
  int tile_begin;    // first linear CTA index of this problem
  const void* bias;  // [Nw] model dtype, or null
  void* out;
  int ldo;
  void* out2;
  int ldo2;
  const void* aux;
  int lda;
  float* ws;         // EPI_PARTIAL: [splits][T][ldw]
  int ldw;
  unsigned long long* best;  // EPI_ARGMAX: [T]
};

struct __align__(64) GemmParams {
  CUtensorMap tmw[kMaxProblems];  // weights, box {64, 128}
  CUtensorMap tmx[kMaxProblems];  // activations, box {64, BN}
  GemmProblem prob[kMaxProblems];
  int nprob;
  int total_tiles;
  DevErr* err;
};

// Plain-pointer view for the SIMT path (fp32 models).
struct SimtGemmParams {
  const void* w[kMaxProblems];
  const void* x[kMaxProblems];
  int ldx[kMaxProblems];
  GemmProblem prob[kMaxProblems];
  int nprob;
  int total_tiles;
};

// ------------------------------------------------------------------ epilogue (per element)
// argmax key: order-preserving bits of the rounded logit above the inverted index, so a
// larger key is a larger value and, among equal values, the lower vocabulary index
// (torch.argmax returns the first maximum).
template <typename T>
ONE_DEVINL unsigned long long argmax_key(float v, int n);
template <>
ONE_DEVINL unsigned long long argmax_key<__nv_bfloat16>(float v, int n) {
  uint32_t b = (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(v));
  b = (b & 0x8000u) ? (~b & 0xFFFFu) : (b | 0x8000u);
  return ((unsigned long long)b << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)n);
}
template <>
ONE_DEVINL unsigned long long argmax_key<float>(float v, int n) {
  uint32_t b = __float_as_uint(v);
  b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return ((unsigned long long)b << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)n);
}

template <typename T>
ONE_DEVINL float bias_at(const GemmProblem& P, int n) {
  return P.bias ? ld<T>(reinterpret_cast<const T*>(P.bias) + n) : 0.0f;
}

// All kinds except GELU_UP / ARGMAX, one (n, t) element. Caller guarantees n < Nw, t < T.
template <typename T>
ONE_DEVINL void epi_elem(const GemmProblem& P, int n, int t, float acc, int split) {
  switch (P.kind) {
    case EPI_STORE: {
      st<T>(reinterpret_cast<T*>(P.out) + (size_t)t * P.ldo + n, acc + bias_at<T>(P, n));
      break;
    }
    case EPI_HXPRE: {
      float y = fminf(fmaxf(rnd<T>(acc + bias_at<T>(P, n)), -100.f), 100.f);
      float a = ld<T>(reinterpret_cast<const T*>(P.aux) + (size_t)t * P.lda + n);
      st<T>(reinterpret_cast<T*>(P.out) + (size_t)t * P.ldo + n, a + y);
      break;
    }
    case EPI_XMOE: {
      float y = fminf(fmaxf(rnd<T>(acc + bias_at<T>(P, n)), -100.f), 100.f);
      float a = ld<T>(reinterpret_cast<const T*>(P.aux) + (size_t)t * P.lda + n);
      st<T>(reinterpret_cast<T*>(P.out) + (size_t)t * P.ldo + n, a * y);
      break;
    }
    case EPI_CX: {
      float y = rnd<T>(acc + bias_at<T>(P, n));
      st<T>(reinterpret_cast<T*>(P.out) + (size_t)t * P.ldo + n, y);
      st<T>(reinterpret_cast<T*>(P.out2) + (size_t)t * P.ldo2 + n, fminf(fmaxf(y, -1e4f), 1e4f));
      break;
    }
    case EPI_PARTIAL: {
      P.ws[((size_t)split * P.T + t) * P.ldw + n] = acc;
      break;
    }
    default:
      break;
  }
}

// OneMLP on an interleaved gate/up weight: packed row 2j is gate_proj row j, 2j+1 is
// up_proj row j. Bias (mlp_bias) is interleaved the same way.
template <typename T>
ONE_DEVINL void epi_gelu_pair(const GemmProblem& P, int n_even, int t, float g, float u) {
  float gb = rnd<T>(g + bias_at<T>(P, n_even));
  float ub = rnd<T>(u + bias_at<T>(P, n_even + 1));
  float a = rnd<T>(gelu_erf(gb));
  st<T>(reinterpret_cast<T*>(P.out) + (size_t)t * P.ldo + (n_even >> 1), a * ub);
}


// ------------------------------------------------------------------ tensor-core kernel
// ST > 0: a deeper ring (more bytes in flight per CTA, one CTA per SM) for launches whose
// CTAs each have an SM to themselves.
template <int BN, int ST = 0>
struct TcCfg {
  // default pipeline depth: keeps two CTAs per SM (<= ~100 KB of stages)
  static constexpr int kStages = ST > 0 ? ST : (BN >= 256 ? 2 : (BN >= 128 ? 3 : 4));
  static constexpr int kABytes = 128 * 64 * 2;
  static constexpr int kBBytes = BN * 64 * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  // the epilogue stages the accumulator through the (drained) pipeline buffers in
  // column chunks of kChunk tokens: kChunk * 128 rows * 4 B must fit in them
  static constexpr int kChunk = (kStages * kStageBytes) / (128 * 4) >= BN ? BN : 128;
  static_assert(kChunk * 128 * 4 <= kStages * kStageBytes, "epilogue staging tile exceeds the pipeline buffers");
  static_assert(BN % kChunk == 0, "token tile must be a multiple of the staging chunk");
  static constexpr int kSmem = kStages * kStageBytes + 1024 /*align*/ + 256 /*barriers*/;
  static constexpr int kThreads = 192;  // w0 TMA, w1 MMA + TMEM owner, w2..5 epilogue
};

// Epilogue of the tensor-core GEMM, run by all six warps (e = 0..191: warps 2..5 first, then
// the TMA and MMA warps once their loops are done).
//   prefetch: right after the dependency wait, each thread loads the bias of its 8-row slice
//             and, for the kinds that read an activation (hx, mean), the aux vectors of its
//             output units into registers, so no global load sits behind the accumulator.
//   E1: warps 2..5 copy their TMEM lane quarter (warp % 4) into a shared fp32 tile
//       S[token][row] (the drained pipeline buffers), kChunk tokens at a time.
//   E2: unit = (token, 8 consecutive rows) [GELU_UP: (token, 8 outputs from 16 rows)];
//       thread e owns the row slice e % 16 (e % 8) of every 12th (24th) token; 16-byte stores.
// Epilogue of 8 consecutive outputs of one token on packed bf16x2 pairs (a = accumulator +
// bias, fp32): y = rnd(a); CX stores y and clamp(y, +-bf16(1e4)); HXPRE stores
// rnd(aux + clamp(y, +-100)), XMOE rnd(aux * clamp(y, +-100)), RESID rnd(aux + y). The bounds are bf16 values and
// each packed add / multiply of bf16 operands is one rounding of the exact result, so the
// values equal the fp32-then-round sequence of one/modeling_one.py:559-565 and
// one/linear_moe.py:53.
// `st` false computes without storing (the epilogue's instruction-cache warm-up pass).
ONE_DEVINL void epi_packed8(int kind, const float (&a)[8], const uint4& aux, __nv_bfloat16* out, __nv_bfloat16* out2,
                            bool st = true) {
  uint32_t y[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) y[j] = pack_bf16x2(a[2 * j], a[2 * j + 1]);
  if (kind == EPI_CX) {
    if (st) *reinterpret_cast<uint4*>(out) = make_uint4(y[0], y[1], y[2], y[3]);
    uint32_t z[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) z[j] = bf2_min(bf2_max(y[j], 0xc61cc61cu), 0x461c461cu);  // +-9984
    if (st) *reinterpret_cast<uint4*>(out2) = make_uint4(z[0], z[1], z[2], z[3]);
    return;
  }
  const uint32_t x[4] = {aux.x, aux.y, aux.z, aux.w};
  uint32_t o[4];
  if (kind == EPI_RESID) {
#pragma unroll
    for (int j = 0; j < 4; ++j) o[j] = bf2_add(x[j], y[j]);
    if (st) *reinterpret_cast<uint4*>(out) = make_uint4(o[0], o[1], o[2], o[3]);
    return;
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t cl = bf2_min(bf2_max(y[j], 0xc2c8c2c8u), 0x42c842c8u);  // +-100
    o[j] = kind == EPI_HXPRE ? bf2_add(x[j], cl) : bf2_mul(x[j], cl);
  }
  if (st) *reinterpret_cast<uint4*>(out) = make_uint4(o[0], o[1], o[2], o[3]);
}

template <int BN>
__device__ __forceinline__ void tc_epilogue(const GemmParams& p, const GemmProblem& P, float* S, uint32_t tmem,
                                            uint64_t* accb, int m_tile, int n_tile, int split) {
  using T = __nv_bfloat16;
  constexpr int CH = TcCfg<BN>::kChunk < 64 ? TcCfg<BN>::kChunk : 64;  // <= 8 prefetched vectors per thread
  constexpr int NT = 192;                 // epilogue threads
  constexpr int TU = NT / 16, TG = NT / 8; // tokens covered per pass: (token, 8-row) / gelu units
  constexpr int KU = (CH + TU - 1) / TU;   // (token, 8-row) units per thread per chunk
  constexpr int KG = (CH + TG - 1) / TG;   // gelu units per thread per chunk
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, q = warp & 3;
  const int e = warp >= 2 ? threadIdx.x - 64 : threadIdx.x + 128;
  const bool drain = warp >= 2;  // owns a TMEM lane quarter
  const int n_base = m_tile * 128;
  const int t_tile = n_tile * BN;
  const int kind = P.kind;
  const bool aux_kind = kind == EPI_HXPRE || kind == EPI_XMOE;
  pdl_wait();
  // ---- prefetch (independent of the accumulator)
  const int c8 = e & 15, n0 = n_base + c8 * 8;
  const bool v8 = n0 < P.Nw;
  float b8[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  if (kind != EPI_GELU_UP && kind != EPI_ARGMAX && kind != EPI_PARTIAL && P.bias && v8)
    load8(reinterpret_cast<const T*>(P.bias) + n0, b8);
  const int cg = e & 7, ng = n_base + cg * 16;
  float bg[16] = {0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0};
  if (kind == EPI_GELU_UP && P.bias && ng < P.Nw) {
    load8(reinterpret_cast<const T*>(P.bias) + ng, bg);
    load8(reinterpret_cast<const T*>(P.bias) + ng + 8, bg + 8);
  }
  uint4 auxr[KU];
#pragma unroll
  for (int k = 0; k < KU; ++k) auxr[k] = make_uint4(0, 0, 0, 0);
  auto aux_load = [&](int cc) {
#pragma unroll
    for (int k = 0; k < KU; ++k) {
      const int t = t_tile + cc + (e >> 4) + TU * k;
      auxr[k] = make_uint4(0, 0, 0, 0);
      if (aux_kind && v8 && t < P.T && (e >> 4) + TU * k < CH)
        auxr[k] = *reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(P.aux) + (size_t)t * P.lda + n0);
    }
  };
  // Two passes over the same code. Pass 0 runs on warps 2..5 while the MMAs are still in flight,
  // with the TMEM reads and every global store switched off: it only brings this code into the
  // instruction cache, where a cold epilogue otherwise spent about a microsecond missing after
  // the accumulator was ready. Pass 1 is the epilogue proper, on all six warps. The first
  // chunk's activation vectors are requested at the start of pass 1, before the accumulator
  // wait: requested before pass 0, they held pass 0 (which computes on them) for a global-load
  // latency, and the warps then met a ready accumulator late (0.6-1 us on the hx and x_moe GEMMs).
  bool ok = true;
#pragma unroll 1
  for (int pass = drain ? 0 : 1; pass < 2; ++pass) {
  const bool dry = pass == 0;
  const int nt = dry ? 128 : NT;  // threads of the pass's named barrier
  const int bar = dry ? 2 : 1;    // its own barrier: warps 0 and 1 may already wait on barrier 1
  if (!dry) {
    aux_load(0);
    ok = mbar_wait(accb, 0, p.err, 3);
    tc_fence_after();
  }
  for (int cc = 0; cc < BN; cc += CH) {
    const int tn = min(CH, P.T - (t_tile + cc));
    if (tn <= 0) break;
    if (cc > 0 && !dry) aux_load(cc);
    // ---- E1
    if (kind == EPI_ARGMAX) {
      if (dry) break;
      // per token: max over this warp's 32 rows of a 32-bit key (order-preserving bf16 bits,
      // then 255 - row in tile, so equal values keep the lowest row), one redux per token;
      // the four warps' keys meet in S, then one 64-bit atomicMax per token and CTA.
      uint32_t* K = reinterpret_cast<uint32_t*>(S);  // [4 warps][CH tokens]
      const int nrow = n_base + q * 32 + lane;
      const int nl = q * 32 + lane;
      T* out = reinterpret_cast<T*>(P.out);
      if (ok && drain)
        for (int c0 = 0; c0 < CH; c0 += 16) {
          if (c0 >= tn) break;  // warp-uniform
          float v[16];
          tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(cc + c0), v);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            uint32_t key = 0u;
            if (nrow < P.Nw) {
              uint32_t b = (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(v[j]));
              b = (b & 0x8000u) ? (~b & 0xFFFFu) : (b | 0x8000u);
              key = (b << 8) | (uint32_t)(255 - nl);
              if (out && c0 + j < tn) st<T>(out + (size_t)(t_tile + cc + c0 + j) * P.ldo + nrow, v[j]);
            }
            key = __reduce_max_sync(0xffffffffu, key);
            if (lane == 0) K[q * CH + c0 + j] = key;
          }
        }
      named_barrier_sync(1, NT);
      for (int tl = e; tl < tn; tl += NT) {
        uint32_t best = 0u;
#pragma unroll
        for (int w = 0; w < 4; ++w) best = max(best, K[w * CH + tl]);
        if (best) {
          const int n = n_base + 255 - (int)(best & 0xFFu);
          const uint32_t b = best >> 8;
          atomicMax(P.best + t_tile + cc + tl,
                    ((unsigned long long)b << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)n));
        }
      }
      named_barrier_sync(1, NT);
      continue;
    }
    if (ok && drain)
      for (int c0 = 0; c0 < CH; c0 += 16) {
        if (c0 >= tn) break;  // warp-uniform
        float v[16];
        if (!dry) {
          tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(cc + c0), v);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 16; ++j) S[(c0 + j) * 128 + q * 32 + lane] = v[j];
        }
      }
    named_barrier_sync(bar, nt);
    // ---- E2
    const int tb = t_tile + cc;
    if (false) {
    } else if (kind == EPI_GELU_UP) {
      T* out = reinterpret_cast<T*>(P.out);
#pragma unroll
      for (int k = 0; k < KG; ++k) {
        const int tl = (e >> 3) + TG * k;
        if (tl >= tn || ng >= P.Nw) continue;
        const float* sv = S + tl * 128 + cg * 16;
        // gelu(g) * u on packed pairs: g, u and gelu(g) rounded to bf16, one rounded product
        uint32_t o4[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint32_t g2 = pack_bf16x2(sv[4 * j] + bg[4 * j], sv[4 * j + 2] + bg[4 * j + 2]);
          const uint32_t u2 = pack_bf16x2(sv[4 * j + 1] + bg[4 * j + 1], sv[4 * j + 3] + bg[4 * j + 3]);
          o4[j] = bf2_mul(pack_bf16x2(gelu_erf(bf2_lo(g2)), gelu_erf(bf2_hi(g2))), u2);
        }
        if (!dry)
          *reinterpret_cast<uint4*>(out + (size_t)(tb + tl) * P.ldo + (ng >> 1)) = make_uint4(o4[0], o4[1], o4[2], o4[3]);
      }
    } else {
#pragma unroll
      for (int k = 0; k < KU; ++k) {
        const int tl = (e >> 4) + TU * k;
        if (tl >= tn || !v8) continue;
        const int t = tb + tl;
        float a[8];
        {
          const float4 f0 = *reinterpret_cast<const float4*>(S + tl * 128 + c8 * 8);
          const float4 f1 = *reinterpret_cast<const float4*>(S + tl * 128 + c8 * 8 + 4);
          a[0] = f0.x; a[1] = f0.y; a[2] = f0.z; a[3] = f0.w; a[4] = f1.x; a[5] = f1.y; a[6] = f1.z; a[7] = f1.w;
        }
        if (kind == EPI_PARTIAL) {
          if (!dry) store8(P.ws + ((size_t)split * P.T + t) * P.ldw + n0, a);
          continue;
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) a[j] += b8[j];
        T* out = reinterpret_cast<T*>(P.out) + (size_t)t * P.ldo + n0;
        if (kind == EPI_STORE) {
          if (!dry) store8(out, a);
        } else {
          epi_packed8(kind, a, auxr[k], out, reinterpret_cast<T*>(P.out2) + (size_t)t * P.ldo2 + n0, !dry);
        }
      }
    }
    named_barrier_sync(bar, nt);
  }
  }
}

// Linear tile index -> (problem, split, m tile, n tile, first k block, k blocks). Token tile
// fastest (m_fast = 0: the CTAs that share a weight slice run together and the slice comes
// from HBM once) for few token tiles; weight tile fastest (m_fast = 1) when the token tiles
// are many, so the CTAs running at once share a few activation slabs in L2 instead of each
// streaming its own slab from HBM once per weight tile.
ONE_DEVINL void gemm_tile_coords(const GemmParams& p, int tile, int& pi, int& m_tile, int& n_tile, int& split, int& kb0,
                                 int& nkb) {
  pi = 0;
  while (pi + 1 < p.nprob && tile >= p.prob[pi + 1].tile_begin) ++pi;
  const GemmProblem& P = p.prob[pi];
  int local = tile - P.tile_begin;
  if (P.m_fast) {
    m_tile = local % P.m_tiles;
    local /= P.m_tiles;
    n_tile = local % P.n_tiles;
    local /= P.n_tiles;
  } else {
    n_tile = local % P.n_tiles;
    local /= P.n_tiles;
    m_tile = local % P.m_tiles;
    local /= P.m_tiles;
  }
  split = local;
  const int kb_total = (P.K + 63) / 64;
  kb0 = split * P.kb_per_split;
  nkb = min(kb0 + P.kb_per_split, kb_total) - kb0;
}

template <int BN, int ST = 0>
__global__ void __launch_bounds__(192, 2) gemm_bf16_tc_kernel(const __grid_constant__ GemmParams p) {
  using C = TcCfg<BN, ST>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kStages * C::kStageBytes);
  uint64_t* empty = full + C::kStages;
  uint64_t* accb = empty + C::kStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accb + 1);

  // linear tile -> (problem, split, m tile, n tile): gemm_tile_coords
  int pi, m_tile, n_tile, split, kb0, nkb;
  gemm_tile_coords(p, blockIdx.x, pi, m_tile, n_tile, split, kb0, nkb);
  const GemmProblem& P = p.prob[pi];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accb, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, BN);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&p.tmw[pi]);
    tma_prefetch_desc(&p.tmx[pi]);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (threadIdx.x == 0) pdl_launch_dependents();

  auto sA = [&](int s) { return smem + s * C::kStageBytes; };
  auto sB = [&](int s) { return smem + s * C::kStageBytes + C::kABytes; };

  if (warp == 0) {
    if (lane == 0) {
      // Weights do not depend on the previous kernel: the first stages are requested, and the
      // rest of the CTA's weight slice is brought into L2, before the dependency wait. The ring
      // refills one slot per consumed k block, so the later weight tiles then come from L2
      // instead of costing an HBM round trip each.
      const uint64_t wpol = l2_policy_evict_first();
      const int pre = min(nkb, C::kStages);
      for (int i = 0; i < pre; ++i) {
        mbar_arrive_expect_tx(&full[i], C::kStageBytes);
        tma_load_2d_hint(sA(i), &p.tmw[pi], &full[i], (kb0 + i) * 64, m_tile * 128, wpol);
      }
      for (int i = pre; i < nkb; ++i) tma_prefetch_l2_2d(&p.tmw[pi], (kb0 + i) * 64, m_tile * 128);
      pdl_wait();
      for (int i = 0; i < nkb; ++i) {
        const int s = i % C::kStages;
        const uint32_t ph = (uint32_t)(i / C::kStages) & 1u;
        if (i >= pre) {
          if (!mbar_wait(&empty[s], ph ^ 1u, p.err, 1)) break;
          mbar_arrive_expect_tx(&full[s], C::kStageBytes);
          tma_load_2d_hint(sA(s), &p.tmw[pi], &full[s], (kb0 + i) * 64, m_tile * 128, wpol);
        }
        tma_load_2d(sB(s), &p.tmx[pi], &full[s], (kb0 + i) * 64, n_tile * BN);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_bf16(128, BN);
      for (int i = 0; i < nkb; ++i) {
        const int s = i % C::kStages;
        const uint32_t ph = (uint32_t)(i / C::kStages) & 1u;
        if (!mbar_wait(&full[s], ph, p.err, 2)) break;
        tc_fence_after();
        const uint64_t ad = umma_desc_sw128(sA(s));
        const uint64_t bd = umma_desc_sw128(sB(s));
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)  // 4 x K=16 per 64-wide stage; +32 B per step
          umma_bf16(tmem, ad + 2 * kk, bd + 2 * kk, idesc, (i | kk) != 0 ? 1u : 0u);
        umma_commit(&empty[s]);
      }
      umma_commit(accb);
    }
  }
  // ---------------- epilogue (all six warps; the TMA / MMA lanes rejoin their warps first)
  __syncwarp();
  tc_epilogue<BN>(p, P, reinterpret_cast<float*>(smem), tmem, accb, m_tile, n_tile, split);
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, BN);
  }
}

// ------------------------------------------------------------------ persistent tensor-core kernel
// Large GEMMs (prompt ingestion, batched LinearMoE): one CTA per SM loops over the tiles
// (tile = blockIdx.x + i * gridDim.x, the linear order above). Warp 0 streams A / B stages
// through a kPStages-deep ring, warp 1 issues the MMAs into one of two TMEM accumulators
// (columns [0, kPBN) and [kPBN, 2 kPBN)), and kPGroups groups of four epilogue warps (2..5,
// 6..9, 10..13, 14..17) drain the other accumulator, taking the kPChunk-token chunks in turn
// (four chunks a group per tile), each group through its own staging tile, so a tile's
// epilogue runs under the next tile's main loop. Same epilogue steps and rounding as
// tc_epilogue (no fused argmax).
constexpr int kPStages = 4;
constexpr int kPBN = 256;
constexpr int kPChunk = 16;  // tokens per staging pass
constexpr int kPGroups = 4;  // epilogue groups of four warps
struct PCfg {
  static constexpr int kABytes = 128 * 64 * 2;
  static constexpr int kBBytes = kPBN * 64 * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kStagingOff = kPStages * kStageBytes;
  static constexpr int kStagingBytes = kPChunk * 128 * 4;  // per epilogue group
  static constexpr int kBarOff = kStagingOff + kPGroups * kStagingBytes;
  static constexpr int kSmem = kBarOff + 256 + 1024 /*align*/;
  static constexpr int kEpiThreads = kPGroups * 128;
  static constexpr int kThreads = 64 + kEpiThreads;  // TMA warp, MMA warp, epilogue groups
};
static_assert(PCfg::kSmem <= 227 * 1024, "persistent GEMM shared memory");

constexpr int kPKU = kPChunk / 8;  // (token, 8-row) units per thread per chunk (128 threads a group)

// The activation operand (hx / mean) of this thread's units in the chunk at token cc of the
// tile: issued one chunk ahead of its use, so its latency hides under the current chunk.
ONE_DEVINL void epi_aux_load(const GemmProblem& P, int m_tile, int n_tile, int cc, int e, uint4 (&aux)[kPKU]) {
  using T = __nv_bfloat16;
  const int n0 = m_tile * 128 + (e & 15) * 8;
  const bool use = (P.kind == EPI_HXPRE || P.kind == EPI_XMOE || P.kind == EPI_RESID) && n0 < P.Nw && cc < kPBN;
#pragma unroll
  for (int k = 0; k < kPKU; ++k) {
    const int t = n_tile * kPBN + cc + (e >> 4) + 8 * k;
    aux[k] = make_uint4(0, 0, 0, 0);
    if (use && t < P.T) aux[k] = *reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(P.aux) + (size_t)t * P.lda + n0);
  }
}

// One tile's epilogue by one group of four warps (group grp: warps 2 + 4 grp .. 5 + 4 grp;
// e = 0..127 within the group): TMEM quarter q = warp % 4, accumulator columns
// [col0, col0 + kPBN); the group takes the chunks cc = (kPGroups j + grp) * kPChunk, staged
// through S.
// aux holds the operands of the group's first chunk (epi_aux_load, issued by the caller).
ONE_DEVINL void tc_epilogue_p(const GemmProblem& P, float* S, uint32_t tmem, uint32_t col0, int m_tile, int n_tile,
                              int split, int grp, uint4 (&aux)[kPKU]) {
  using T = __nv_bfloat16;
  constexpr int CH = kPChunk, NT = 128;
  constexpr int TU = NT / 16, TG = NT / 8;  // tokens per pass: (token, 8-row) / gelu units
  constexpr int KU = CH / TU, KG = CH / TG;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, q = warp & 3;
  const int e = threadIdx.x - 64 - 128 * grp;
  const int bar = 1 + grp;
  const int n_base = m_tile * 128, t_tile = n_tile * kPBN;
  const int kind = P.kind;
  const bool aux_kind = kind == EPI_HXPRE || kind == EPI_XMOE || kind == EPI_RESID;
  const int c8 = e & 15, n0 = n_base + c8 * 8;
  const bool v8 = n0 < P.Nw;
  float b8[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  if (kind != EPI_GELU_UP && kind != EPI_PARTIAL && P.bias && v8) load8(reinterpret_cast<const T*>(P.bias) + n0, b8);
  const int cg = e & 7, ng = n_base + cg * 16;
  float bg[16] = {0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0};
  if (kind == EPI_GELU_UP && P.bias && ng < P.Nw) {
    load8(reinterpret_cast<const T*>(P.bias) + ng, bg);
    load8(reinterpret_cast<const T*>(P.bias) + ng + 8, bg + 8);
  }
  static_assert(KU == kPKU, "aux prefetch shape");
  for (int cc = grp * CH; cc < kPBN; cc += kPGroups * CH) {
    const int tn = min(CH, P.T - (t_tile + cc));
    if (tn <= 0) break;
    uint4 auxr[KU];
#pragma unroll
    for (int k = 0; k < KU; ++k) auxr[k] = aux[k];
    if (aux_kind) epi_aux_load(P, m_tile, n_tile, cc + kPGroups * CH, e, aux);  // next chunk
    // ---- E1: this warp's TMEM lane quarter -> S[token][row]
#pragma unroll
    for (int c0 = 0; c0 < CH; c0 += 16) {
      if (c0 >= tn) break;  // warp-uniform
      float v[16];
      tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + col0 + (uint32_t)(cc + c0), v);
      tmem_ld_wait();
#pragma unroll
      for (int j = 0; j < 16; ++j) S[(c0 + j) * 128 + q * 32 + lane] = v[j];
    }
    named_barrier_sync(bar, NT);
    // ---- E2
    const int tb = t_tile + cc;
    if (kind == EPI_GELU_UP) {
      T* out = reinterpret_cast<T*>(P.out);
#pragma unroll
      for (int k = 0; k < KG; ++k) {
        const int tl = (e >> 3) + TG * k;
        if (tl >= tn || ng >= P.Nw) continue;
        const float* sv = S + tl * 128 + cg * 16;
        // gelu(g) * u on packed pairs: g, u and gelu(g) rounded to bf16, one rounded product
        uint32_t o4[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint32_t g2 = pack_bf16x2(sv[4 * j] + bg[4 * j], sv[4 * j + 2] + bg[4 * j + 2]);
          const uint32_t u2 = pack_bf16x2(sv[4 * j + 1] + bg[4 * j + 1], sv[4 * j + 3] + bg[4 * j + 3]);
          o4[j] = bf2_mul(pack_bf16x2(gelu_erf(bf2_lo(g2)), gelu_erf(bf2_hi(g2))), u2);
        }
        *reinterpret_cast<uint4*>(out + (size_t)(tb + tl) * P.ldo + (ng >> 1)) = make_uint4(o4[0], o4[1], o4[2], o4[3]);
      }
    } else {
#pragma unroll
      for (int k = 0; k < KU; ++k) {
        const int tl = (e >> 4) + TU * k;
        if (tl >= tn || !v8) continue;
        const int t = tb + tl;
        float a[8];
        {
          const float4 f0 = *reinterpret_cast<const float4*>(S + tl * 128 + c8 * 8);
          const float4 f1 = *reinterpret_cast<const float4*>(S + tl * 128 + c8 * 8 + 4);
          a[0] = f0.x; a[1] = f0.y; a[2] = f0.z; a[3] = f0.w; a[4] = f1.x; a[5] = f1.y; a[6] = f1.z; a[7] = f1.w;
        }
        if (kind == EPI_PARTIAL) {
          store8(P.ws + ((size_t)split * P.T + t) * P.ldw + n0, a);
          continue;
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) a[j] += b8[j];
        T* out = reinterpret_cast<T*>(P.out) + (size_t)t * P.ldo + n0;
        if (kind == EPI_STORE) {
          store8(out, a);
        } else {
          epi_packed8(kind, a, auxr[k], out, reinterpret_cast<T*>(P.out2) + (size_t)t * P.ldo2 + n0);
        }
      }
    }
    named_barrier_sync(bar, NT);
  }
}

__global__ void __launch_bounds__(PCfg::kThreads, 1) gemm_bf16_tc_persistent(const __grid_constant__ GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + PCfg::kBarOff);
  uint64_t* empty = full + kPStages;
  uint64_t* accf = empty + kPStages;  // [2] accumulator b holds a finished tile
  uint64_t* acce = accf + 2;          // [2] accumulator b drained by the epilogue
  uint64_t* drain = acce + 2;         // the MMA thread's last commit
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  int* eflag = reinterpret_cast<int*>(tmem_slot + 1);  // [4 kPGroups] epilogue warps' wait results
  float* S = reinterpret_cast<float*>(smem + PCfg::kStagingOff);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kPStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&accf[b], 1);
      mbar_init(&acce[b], PCfg::kEpiThreads);
    }
    mbar_init(drain, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 2 * kPBN);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0)
    for (int i = 0; i < p.nprob; ++i) {
      tma_prefetch_desc(&p.tmw[i]);
      tma_prefetch_desc(&p.tmx[i]);
    }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (threadIdx.x == 0) pdl_launch_dependents();
  auto sA = [&](int s) { return smem + s * PCfg::kStageBytes; };
  auto sB = [&](int s) { return smem + s * PCfg::kStageBytes + PCfg::kABytes; };

  if (warp == 0) {
    if (lane == 0) {
      pdl_wait();
      int it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < p.total_tiles; tile += gridDim.x) {
        int pi, m_tile, n_tile, split, kb0, nkb;
        gemm_tile_coords(p, tile, pi, m_tile, n_tile, split, kb0, nkb);
        for (int i = 0; i < nkb; ++i, ++it) {
          const int s = it % kPStages;
          const uint32_t ph = (uint32_t)(it / kPStages) & 1u;
          if (!mbar_wait(&empty[s], ph ^ 1u, p.err, 21)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[s], PCfg::kStageBytes);
          tma_load_2d(sA(s), &p.tmw[pi], &full[s], (kb0 + i) * 64, m_tile * 128);
          tma_load_2d(sB(s), &p.tmx[pi], &full[s], (kb0 + i) * 64, n_tile * kPBN);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_bf16(128, kPBN);
      int it = 0, ti = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < p.total_tiles; tile += gridDim.x, ++ti) {
        int pi, m_tile, n_tile, split, kb0, nkb;
        gemm_tile_coords(p, tile, pi, m_tile, n_tile, split, kb0, nkb);
        const int b = ti & 1;
        if (!mbar_wait(&acce[b], ((uint32_t)(ti >> 1) & 1u) ^ 1u, p.err, 22)) break;
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(b * kPBN);
        for (int i = 0; i < nkb; ++i, ++it) {
          const int s = it % kPStages;
          const uint32_t ph = (uint32_t)(it / kPStages) & 1u;
          if (!mbar_wait(&full[s], ph, p.err, 23)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t ad = umma_desc_sw128(sA(s));
          const uint64_t bd = umma_desc_sw128(sB(s));
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) umma_bf16(d, ad + 2 * kk, bd + 2 * kk, idesc, (i | kk) != 0 ? 1u : 0u);
          umma_commit(&empty[s]);
        }
        if (ok) umma_commit(&accf[b]);
      }
      // every MMA issued by this thread has completed before the teardown frees TMEM
      umma_commit(drain);
      mbar_wait(drain, 0, p.err, 24);
    }
  } else {
    pdl_wait();
    int ti = 0;
    for (int tile = blockIdx.x; tile < p.total_tiles; tile += gridDim.x, ++ti) {
      int pi, m_tile, n_tile, split, kb0, nkb;
      gemm_tile_coords(p, tile, pi, m_tile, n_tile, split, kb0, nkb);
      const int b = ti & 1;
      // the first chunk's activation operands are requested before the accumulator wait
      const int grp = (warp - 2) >> 2;
      uint4 aux[kPKU];
      epi_aux_load(p.prob[pi], m_tile, n_tile, grp * kPChunk, threadIdx.x - 64 - 128 * grp, aux);
      // one waiter per warp; the epilogue warps agree before they leave together
      bool ok = true;
      if (lane == 0) ok = mbar_wait(&accf[b], (uint32_t)(ti >> 1) & 1u, p.err, 25);
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      if (lane == 0) eflag[warp - 2] = ok ? 1 : 0;
      named_barrier_sync(1 + kPGroups, PCfg::kEpiThreads);
      bool all_ok = true;
#pragma unroll
      for (int w = 0; w < 4 * kPGroups; ++w) all_ok = all_ok && eflag[w];
      named_barrier_sync(1 + kPGroups, PCfg::kEpiThreads);
      if (!all_ok) break;
      tc_fence_after();
      tc_epilogue_p(p.prob[pi], S + grp * (PCfg::kStagingBytes / 4), tmem, (uint32_t)(b * kPBN), m_tile, n_tile, split,
                    grp, aux);
      tc_fence_before();
      mbar_arrive(&acce[b]);
    }
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 2 * kPBN);
  }
}

// ------------------------------------------------------------------ SIMT kernel (fp32 models)
// 64 weight rows x 64 tokens per CTA, 256 threads, 4x4 outputs per thread, K staged in
// shared memory 16 at a time. Rows of a thread are 4 consecutive n, so an interleaved
// gate/up pair always sits in one thread.
template <typename T>
__global__ void __launch_bounds__(256) gemm_simt_kernel(const SimtGemmParams p, DevErr* err) {
  __shared__ float sW[16][65];
  __shared__ float sX[16][65];
  pdl_wait();
  const int tile = blockIdx.x;
  int pi = 0;
  while (pi + 1 < p.nprob && tile >= p.prob[pi + 1].tile_begin) ++pi;
  const GemmProblem& P = p.prob[pi];
  int local = tile - P.tile_begin;
  const int n_tile = local % P.n_tiles;
  local /= P.n_tiles;
  const int m_tile = local % P.m_tiles;
  const int split = local / P.m_tiles;
  const int k0 = split * P.kb_per_split * 64;
  const int k1 = min(P.K, k0 + P.kb_per_split * 64);
  const T* W = reinterpret_cast<const T*>(p.w[pi]);
  const T* X = reinterpret_cast<const T*>(p.x[pi]);
  const int ldx = p.ldx[pi];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;  // ty: rows, tx: tokens
  const int nb = m_tile * 64, tb = n_tile * 64;
  float acc[4][4] = {};
  for (int kk = k0; kk < k1; kk += 16) {
    for (int i = threadIdx.x; i < 16 * 64; i += 256) {
      const int r = i >> 4, c = i & 15;
      const int n = nb + r, t = tb + r, k = kk + c;
      sW[c][r] = (n < P.Nw && k < k1) ? ld<T>(W + (size_t)n * P.K + k) : 0.f;
      sX[c][r] = (t < P.T && k < k1) ? ld<T>(X + (size_t)t * ldx + k) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int c = 0; c < 16; ++c) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        a[i] = sW[c][ty * 4 + i];
        b[i] = sX[c][tx * 4 + i];
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int n = nb + ty * 4 + i;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int t = tb + tx * 4 + j;
      if (n >= P.Nw || t >= P.T) continue;
      if (P.kind == EPI_GELU_UP) {
        if (!(i & 1)) epi_gelu_pair<T>(P, n, t, acc[i][j], acc[i + 1][j]);
      } else if (P.kind == EPI_ARGMAX) {
        if (P.out) st<T>(reinterpret_cast<T*>(P.out) + (size_t)t * P.ldo + n, acc[i][j]);
        atomicMax(P.best + t, argmax_key<T>(acc[i][j], n));
      } else {
        epi_elem<T>(P, n, t, acc[i][j], split);
      }
    }
  }
}

}  // namespace one

namespace one {

// ------------------------------------------------------------------ lm_head with fused argmax
// logits[t, v] = rnd(sum_k X[t, k] * W[v, k]) for a [T, K] activation and the [V, K] tied
// embedding (one/modeling_one.py:902), with each token's greedy choice (the first maximum over
// v of the rounded logits, torch.argmax) reduced into best[t] as an order-preserving 64-bit key
// by atomicMax (argmax_key). Written only on request: the logits themselves.
//
// Tokens are the UMMA A operand (M = 128 token rows per tile) and a 224-row vocabulary tile is
// B (N = 224), so TMEM lane i holds token i's 224 logits of the tile: each epilogue thread scans
// its own row in vocabulary order and needs no cross-thread reduction. One CTA per (vocabulary
// tile, pair of token tiles): both token tiles of a decode step (256 tokens) multiply the same
// vocabulary tile into two TMEM accumulators (256 columns apart), so the 143 vocabulary tiles of
// a 32000-word head run as one wave of 143 CTAs on the 148 SMs (a CTA per token tile made two
// waves; 256-row tiles left 23 SMs idle with 8/7 of the work on the others).
// One thread's bulk copies complete one after another (~0.4 us each on B200), so every copy of
// a ring slot has its own issuing thread: lane 0 of warp 2 + 3 s streams slot s's vocabulary
// tiles (the first before the dependency wait), lanes 0 of warps 3 + 3 s and 4 + 3 s its two
// token tiles. Warp 1 issues the MMAs; warps 2..9 scan the accumulators, one token tile per
// warp and 32 of its tokens (TMEM lane quarter warp % 4).
constexpr int kLmStages = 3;
constexpr int kLmBN = 224;  // vocabulary rows per tile (MMA N: a multiple of 16, <= 256)
constexpr int kLmTT = 2;    // token tiles per CTA
constexpr int kLmAcc = 256; // TMEM columns per token tile's accumulator (power-of-two allocation)
static_assert(kLmBN <= kLmAcc && kLmBN % 32 == 0, "lm_head tile: accumulator columns, 32-column scan");
constexpr int kLmCopies = 1 + kLmTT;  // bulk copies per ring slot
struct LmCfg {
  static constexpr int kABytes = 128 * 64 * 2;    // one token tile
  static constexpr int kBBytes = kLmBN * 64 * 2;  // vocabulary tile
  static constexpr int kStageBytes = kLmTT * kABytes + kBBytes;
  static constexpr int kSmem = kLmStages * kStageBytes + 1024 + 256;
  static constexpr int kIssueWarps = kLmStages * kLmCopies;
  static constexpr int kScanWarps = 4 * kLmTT;
  static constexpr int kThreads = 32 * (2 + (kIssueWarps > kScanWarps ? kIssueWarps : kScanWarps));
};
static_assert(LmCfg::kSmem <= 227 * 1024, "lm_head shared memory");

struct __align__(64) LmParams {
  CUtensorMap tmx;  // activations [T, K], box {64, 128}
  CUtensorMap tmw;  // weights [V, K], box {64, kLmBN}
  int T, V, K;
  int t_tiles;      // token tiles
  __nv_bfloat16* logits;  // [T, ldo] or null
  int ldo;
  unsigned long long* best;  // [T]
  DevErr* err;
};

__global__ void __launch_bounds__(LmCfg::kThreads, 1) lm_head_argmax_kernel(const __grid_constant__ LmParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kLmStages * LmCfg::kStageBytes);
  uint64_t* empty = full + kLmStages;
  uint64_t* accb = empty + kLmStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accb + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t_pairs = (p.t_tiles + kLmTT - 1) / kLmTT;
  const int v_tile = blockIdx.x / t_pairs, tt0 = (blockIdx.x % t_pairs) * kLmTT;
  const int ntt = min(kLmTT, p.t_tiles - tt0);  // token tiles of this CTA
  const int nkb = (p.K + 63) / 64;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kLmStages; ++s) {
      mbar_init(&full[s], 1 + ntt);  // the weight copy and each token-tile copy of the slot arrive
      mbar_init(&empty[s], 1);
    }
    mbar_init(accb, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kLmTT * kLmAcc);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&p.tmx);
    tma_prefetch_desc(&p.tmw);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (threadIdx.x == 0) pdl_launch_dependents();
  auto sA = [&](int s, int tt) { return smem + s * LmCfg::kStageBytes + tt * LmCfg::kABytes; };
  auto sB = [&](int s) { return smem + s * LmCfg::kStageBytes + kLmTT * LmCfg::kABytes; };

  if (warp >= 2 && warp < 2 + LmCfg::kIssueWarps) {
    // TMA issue, one thread per copy of a slot, for the k blocks slot, slot + S, ...
    // (S = kLmStages), before the warp turns to the epilogue
    if (lane == 0) {
      const int slot = (warp - 2) / kLmCopies, cp = (warp - 2) % kLmCopies;
      if (cp == 0) {
        // vocabulary tiles: never written by earlier kernels, so no dependency wait
        const uint64_t wpol = l2_policy_evict_first();
        for (int i = slot; i < nkb; i += kLmStages) {
          const uint32_t ph = (uint32_t)(i / kLmStages) & 1u;
          if (i >= kLmStages && !mbar_wait(&empty[slot], ph ^ 1u, p.err, 41)) break;
          mbar_arrive_expect_tx(&full[slot], LmCfg::kBBytes);
          tma_load_2d_hint(sB(slot), &p.tmw, &full[slot], i * 64, v_tile * kLmBN, wpol);
        }
      } else if (cp - 1 < ntt) {
        // token tile cp - 1: the activations the previous kernel wrote
        const int tt = cp - 1;
        pdl_wait();
        for (int i = slot; i < nkb; i += kLmStages) {
          const uint32_t ph = (uint32_t)(i / kLmStages) & 1u;
          if (i >= kLmStages && !mbar_wait(&empty[slot], ph ^ 1u, p.err, 44)) break;
          mbar_arrive_expect_tx(&full[slot], LmCfg::kABytes);
          tma_load_2d(sA(slot, tt), &p.tmx, &full[slot], i * 64, (tt0 + tt) * 128);
        }
      }
    }
    __syncwarp();
  }
  if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_bf16(128, kLmBN);
      for (int i = 0; i < nkb; ++i) {
        const int s = i % kLmStages;
        const uint32_t ph = (uint32_t)(i / kLmStages) & 1u;
        if (!mbar_wait(&full[s], ph, p.err, 42)) break;
        tc_fence_after();
        const uint64_t bd = umma_desc_sw128(sB(s));
        for (int tt = 0; tt < ntt; ++tt) {
          const uint64_t ad = umma_desc_sw128(sA(s, tt));
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_bf16(tmem + (uint32_t)(tt * kLmAcc), ad + 2 * kk, bd + 2 * kk, idesc, (i | kk) != 0 ? 1u : 0u);
        }
        umma_commit(&empty[s]);
      }
      umma_commit(accb);
    }
  } else if (warp >= 2 && warp < 2 + LmCfg::kScanWarps && (warp - 2) / 4 < ntt) {
    // ---- epilogue: warp w scans token tile (w - 2) / 4, TMEM lanes 32 (w % 4) .. +31 = its
    // 32 tokens of that tile
    pdl_wait();
    const int q = warp & 3;
    const bool ok = mbar_wait(accb, 0, p.err, 43);
    tc_fence_after();
    const int v0 = v_tile * kLmBN;
    {
    const int tt = (warp - 2) / 4;
    const int t = (tt0 + tt) * 128 + q * 32 + lane;
    uint32_t best16 = 0u;  // order-preserving bf16 bits of the best rounded logit (0: none)
    int best_v = 0;
    if (ok) {
      for (int c0 = 0; c0 < kLmBN; c0 += 32) {
        if (v0 + c0 >= p.V) break;  // warp-uniform
        float v[32];
        tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(tt * kLmAcc + c0), v);
        tmem_ld_wait();
        uint32_t h[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) h[j] = pack_bf16x2(v[2 * j], v[2 * j + 1]);
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          uint32_t b = (j & 1) ? (h[j >> 1] >> 16) : (h[j >> 1] & 0xFFFFu);
          b = (b & 0x8000u) ? (~b & 0xFFFFu) : (b | 0x8000u);
          if (v0 + c0 + j < p.V && b > best16) {  // strictly greater: the first maximum wins
            best16 = b;
            best_v = v0 + c0 + j;
          }
        }
        if (p.logits && t < p.T) {
          __nv_bfloat16* dst = p.logits + (size_t)t * p.ldo + v0 + c0;
          if (v0 + c0 + 32 <= p.V && ((reinterpret_cast<uintptr_t>(dst) & 15) == 0)) {
#pragma unroll
            for (int j = 0; j < 4; ++j)
              reinterpret_cast<uint4*>(dst)[j] = make_uint4(h[4 * j], h[4 * j + 1], h[4 * j + 2], h[4 * j + 3]);
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (v0 + c0 + j < p.V)
                dst[j] = __ushort_as_bfloat16((unsigned short)((j & 1) ? (h[j >> 1] >> 16) : (h[j >> 1] & 0xFFFFu)));
          }
        }
      }
    }
    if (ok && t < p.T && best16)
      atomicMax(p.best + t, ((unsigned long long)best16 << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)best_v));
    }
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kLmTT * kLmAcc);
  }
}

}  // namespace one
