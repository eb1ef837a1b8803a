// Exact softmax attention on the 5th-generation tensor cores (tcgen05) for head_dim 64 in
// bf16, and the RoPE prologue of the fused RoPE + attention operator.
//
// Semantics: out = softmax(q k^T * scale [+ causal mask]) v with an fp32 softmax, the
// exact attention of turbo_flash_attention's PyTorch path (one/turbo_ops.py:115-143) and of
// flash_attention()'s exact branch (one/flash_attention.py:242-282). The causal mask is
// top-left aligned (torch.triu(..., diagonal=1)): query i sees keys 0..i.
//
// One CTA takes two 128-row query tiles of one (batch, head) and streams the head's keys
// in 128-key tiles. Twelve warps in three warpgroups:
//   warps 0-3, 4-7   softmax warpgroups, one per query tile, one thread per query row:
//                      S row from TMEM (128 fp32 registers) -> running max ->
//                      p = 2^(s*scale*log2e - m) -> bf16 P row back into TMEM
//   warp 8           TMA producer: Q tiles once, then K and V tiles through a 3-stage ring
//   warp 9           allocates TMEM; one thread issues tcgen05.mma:
//                      S_t = Q_t K_j^T   (M 128, N 128, K 64; both operands K-major in smem)
//                      O_t += P_t V_j    (M 128, N 64, K 128; P read from TMEM, V MN-major)
//   warps 10-11      idle
// The third warpgroup gives up registers (setmaxnreg) so the softmax threads can hold a
// whole score row: 168 per thread at launch, 208 for softmax, 88 for the rest.
// TMEM columns (512): S_0 [0,128), S_1 [128,256), O_0 [256,320), O_1 [320,384),
// P_0 [384,448), P_1 [448,512) (bf16 pairs, one 32-bit column per two keys). A softmax thread releases S_t as soon as the row is in registers, so the
// MMA thread computes S_t for key tile j + 1 while softmax t works on tile j; the two
// query tiles interleave on the tensor core.
//
// The running max is rescaled lazily: O and the row sum are multiplied by 2^(m_old-m_new)
// only when the max has grown by more than 2^8; otherwise p keeps the older, smaller
// max and stays below 2^8, which fp32 accumulators and bf16 P hold exactly as well. The
// final division uses the same max, so the result is the exact softmax either way.
//
// Every wait is bounded (mbar_wait): on timeout the warp records ERR_WAIT_TIMEOUT and
// falls through to teardown, where the producer waits for its copies in flight and the MMA
// thread for its MMAs before TMEM is freed.
#pragma once

namespace one {

constexpr int kFaRows = 128;   // query rows per tile (UMMA M)
constexpr int kFaKeys = 128;   // keys per K / V tile
constexpr int kFaDh = 64;      // head dim handled by the tensor-core kernel
constexpr int kFaQTiles = 2;   // query tiles per CTA
constexpr int kFaStages = 3;   // K / V ring depth
constexpr int kFaThreads = 128 * (kFaQTiles + 1);
constexpr int kFaProducerWarp = 4 * kFaQTiles;
constexpr int kFaMmaWarp = kFaProducerWarp + 1;
// Registers: 65536 per SM in four sub-partitions of 16384; 12 warps -> 3 per sub-partition
// -> 168 per thread at launch. setmaxnreg moves 80 per thread from the third warpgroup to
// the two softmax warpgroups (40 each); the MMA and TMA code needs 88 without spilling.
constexpr int kFaRegsLaunch = 168;
constexpr int kFaRegsSoftmax = 208;
constexpr int kFaRegsOther = 88;
static_assert(kFaQTiles * 128 * kFaRegsSoftmax + 128 * kFaRegsOther <= kFaThreads * kFaRegsLaunch,
              "register split exceeds the launch allocation");
constexpr uint32_t kFaTile = kFaRows * kFaDh * 2;     // one Q, K or V tile: 16 KB
constexpr uint32_t kFaTmemCols = 512;
constexpr uint32_t kFaOffQ = 0;
constexpr uint32_t kFaOffK = kFaOffQ + kFaQTiles * kFaTile;
constexpr uint32_t kFaOffV = kFaOffK + kFaStages * kFaTile;
constexpr uint32_t kFaOffBar = kFaOffV + kFaStages * kFaTile;
// barriers: q_full, k_full[S], k_empty[S], v_full[S], v_empty[S], s_full[Q], s_free[Q],
// p_full[Q], o_full[Q], done
constexpr int kFaBarQ = 0;
constexpr int kFaBarKF = 1;
constexpr int kFaBarKE = kFaBarKF + kFaStages;
constexpr int kFaBarVF = kFaBarKE + kFaStages;
constexpr int kFaBarVE = kFaBarVF + kFaStages;
constexpr int kFaBarSF = kFaBarVE + kFaStages;
constexpr int kFaBarSE = kFaBarSF + kFaQTiles;
constexpr int kFaBarPF = kFaBarSE + kFaQTiles;
constexpr int kFaBarOF = kFaBarPF + kFaQTiles;
constexpr int kFaBarDone = kFaBarOF + kFaQTiles;
constexpr int kFaBars = kFaBarDone + 1;
constexpr size_t kFaSmem = kFaOffBar + kFaBars * 8 + 16 + 1024;  // + TMEM slot + 1 KB alignment slack
static_assert(kFaSmem <= 227 * 1024, "attention tile ring exceeds shared memory");
static_assert(kFaOffK % 1024 == 0 && kFaOffV % 1024 == 0, "swizzled tiles need 1 KB alignment");
constexpr uint32_t kFaColS = 0, kFaColO = kFaQTiles * kFaKeys, kFaColP = kFaColO + kFaQTiles * kFaDh;
static_assert(kFaColP + kFaQTiles * kFaKeys / 2 <= kFaTmemCols, "TMEM columns");

struct FaParams {
  CUtensorMap tq, tk, tv;  // [bh][n][64] bf16, box {64, 128, 1}, 128-byte swizzle, zero fill
  __nv_bfloat16* out;      // [bh][nq][64]
  int nq, nk, causal;
  float scale_log2;        // softmax scale * log2(e)
  DevErr* err;
};

// Key tiles a 128-row query tile starting at q_row0 needs (0 for a tile past the end).
ONE_DEVINL int fa_key_tiles(int q_row0, int nq, int nk, int causal) {
  if (q_row0 >= nq) return 0;
  int n = (nk + kFaKeys - 1) / kFaKeys;
  if (causal) n = min(n, min(q_row0 + kFaRows - 1, nq - 1) / kFaKeys + 1);
  return n;
}

template <int N>
ONE_DEVINL void setmaxnreg_inc() { asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N)); }
template <int N>
ONE_DEVINL void setmaxnreg_dec() { asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N)); }

__global__ void __launch_bounds__(kFaThreads, 1) flash_attn_tc_kernel(const __grid_constant__ FaParams p) {
  extern __shared__ uint8_t fa_smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(fa_smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + kFaOffBar);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + kFaBars);
  pdl_wait();  // inputs written by the previous launch are visible after this
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = blockIdx.x;
  // heaviest query tiles (most keys under a causal mask) launch first
  const int q0 = (gridDim.y - 1 - blockIdx.y) * (kFaRows * kFaQTiles);
  int nkt[kFaQTiles];
  int nkt_max = 0;
#pragma unroll
  for (int t = 0; t < kFaQTiles; ++t) {
    nkt[t] = fa_key_tiles(q0 + t * kFaRows, p.nq, p.nk, p.causal);
    nkt_max = max(nkt_max, nkt[t]);
  }

  if (threadIdx.x == 0) {
    mbar_init(&bar[kFaBarQ], 1);
    for (int s = 0; s < kFaStages; ++s) {
      mbar_init(&bar[kFaBarKF + s], 1);
      mbar_init(&bar[kFaBarKE + s], 1);
      mbar_init(&bar[kFaBarVF + s], 1);
      mbar_init(&bar[kFaBarVE + s], 1);
    }
    for (int t = 0; t < kFaQTiles; ++t) {
      mbar_init(&bar[kFaBarSF + t], 1);
      mbar_init(&bar[kFaBarSE + t], 4);
      mbar_init(&bar[kFaBarPF + t], 4);
      mbar_init(&bar[kFaBarOF + t], 1);
    }
    mbar_init(&bar[kFaBarDone], 1);
    fence_barrier_init();
  }
  if (warp == kFaMmaWarp) {
    tmem_alloc(tmem_slot, kFaTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp >= kFaProducerWarp) {
    setmaxnreg_dec<kFaRegsOther>();
    if (warp == kFaProducerWarp && lane == 0) {
      // ------------------------------------------------------------ TMA producer
      tma_prefetch_desc(&p.tq);
      tma_prefetch_desc(&p.tk);
      tma_prefetch_desc(&p.tv);
      int ntiles = 0;
#pragma unroll
      for (int t = 0; t < kFaQTiles; ++t) ntiles += nkt[t] > 0 ? 1 : 0;
      mbar_arrive_expect_tx(&bar[kFaBarQ], ntiles * kFaTile);
      for (int t = 0; t < ntiles; ++t) tma_load_3d(sm + kFaOffQ + t * kFaTile, &p.tq, &bar[kFaBarQ], 0, q0 + t * kFaRows, bh);
      int issued = 0;
      for (int j = 0; j < nkt_max; ++j) {
        const int s = j % kFaStages;
        const uint32_t ph = (j / kFaStages) & 1;
        if (!mbar_wait(&bar[kFaBarKE + s], ph ^ 1, p.err, 1)) break;
        mbar_arrive_expect_tx(&bar[kFaBarKF + s], kFaTile);
        tma_load_3d(sm + kFaOffK + s * kFaTile, &p.tk, &bar[kFaBarKF + s], 0, j * kFaKeys, bh);
        if (!mbar_wait(&bar[kFaBarVE + s], ph ^ 1, p.err, 2)) {
          mbar_wait(&bar[kFaBarKF + s], ph, p.err, 3);  // the K copy just issued lands before teardown
          break;
        }
        mbar_arrive_expect_tx(&bar[kFaBarVF + s], kFaTile);
        tma_load_3d(sm + kFaOffV + s * kFaTile, &p.tv, &bar[kFaBarVF + s], 0, j * kFaKeys, bh);
        issued = j + 1;
      }
      // copies in flight land before teardown (already complete on the normal path)
      mbar_wait(&bar[kFaBarQ], 0, p.err, 4);
      for (int j = max(0, issued - kFaStages); j < issued; ++j) {
        const int s = j % kFaStages;
        const uint32_t ph = (j / kFaStages) & 1;
        mbar_wait(&bar[kFaBarKF + s], ph, p.err, 5);
        mbar_wait(&bar[kFaBarVF + s], ph, p.err, 6);
      }
    } else if (warp == kFaMmaWarp && lane == 0) {
      // ------------------------------------------------------------ MMA issuer
      constexpr uint32_t idesc_s = umma_idesc_bf16(kFaRows, kFaKeys);
      constexpr uint32_t idesc_o = umma_idesc_bf16_bmn(kFaRows, kFaDh);
      // S_t = Q_t K_j^T (4 MMAs of K 16) and O_t += P_t V_j (8 MMAs of K 16; P advances 8
      // TMEM columns and V 2 KB per 16 keys)
      auto issue_s = [&](int t, int s) {
        const uint64_t a = umma_desc_sw128(sm + kFaOffQ + t * kFaTile);
        const uint64_t b = umma_desc_sw128(sm + kFaOffK + s * kFaTile);
#pragma unroll
        for (int kk = 0; kk < kFaDh / 16; ++kk)
          umma_bf16(tmem + kFaColS + t * kFaKeys, a + 2 * kk, b + 2 * kk, idesc_s, kk > 0 ? 1u : 0u);
        umma_commit(&bar[kFaBarSF + t]);
      };
      auto issue_pv = [&](int t, int s, bool acc) {
        const uint64_t b = umma_desc_sw128_mn(sm + kFaOffV + s * kFaTile, kFaTile);
#pragma unroll
        for (int kk = 0; kk < kFaKeys / 16; ++kk)
          umma_bf16_ta(tmem + kFaColO + t * kFaDh, tmem + kFaColP + t * (kFaKeys / 2) + kk * 8,
                       b + (uint64_t)(kk * (2048 >> 4)), idesc_o, (acc || kk > 0) ? 1u : 0u);
        umma_commit(&bar[kFaBarOF + t]);
      };
      bool ok = mbar_wait(&bar[kFaBarQ], 0, p.err, 7);
      if (ok && nkt_max > 0 && (ok = mbar_wait(&bar[kFaBarKF], 0, p.err, 8))) {
        tc_fence_after();
#pragma unroll
        for (int t = 0; t < kFaQTiles; ++t)
          if (nkt[t] > 0) issue_s(t, 0);
        umma_commit(&bar[kFaBarKE]);
      }
      // per key tile j: S_t for tile j + 1 as soon as softmax t holds S_t(j) in registers,
      // then O_t += P_t V_j as soon as softmax t has written P_t(j)
      for (int j = 0; ok && j < nkt_max; ++j) {
        const int s = j % kFaStages, s1 = (j + 1) % kFaStages;
        if (j + 1 < nkt_max) {
          if (!(ok = mbar_wait(&bar[kFaBarKF + s1], ((j + 1) / kFaStages) & 1, p.err, 9))) break;
#pragma unroll
          for (int t = 0; t < kFaQTiles; ++t) {
            if (j + 1 >= nkt[t]) continue;
            if (!(ok = mbar_wait(&bar[kFaBarSE + t], j & 1, p.err, 10))) break;
            tc_fence_after();
            issue_s(t, s1);
          }
          if (!ok) break;
          umma_commit(&bar[kFaBarKE + s1]);
        }
        if (!(ok = mbar_wait(&bar[kFaBarVF + s], (j / kFaStages) & 1, p.err, 11))) break;
#pragma unroll
        for (int t = 0; t < kFaQTiles; ++t) {
          if (j >= nkt[t]) continue;
          if (!(ok = mbar_wait(&bar[kFaBarPF + t], j & 1, p.err, 12))) break;
          tc_fence_after();
          issue_pv(t, s, j > 0);
        }
        if (!ok) break;
        umma_commit(&bar[kFaBarVE + s]);
      }
      // every MMA issued above completes before TMEM is freed
      umma_commit(&bar[kFaBarDone]);
      mbar_wait(&bar[kFaBarDone], 0, p.err, 13);
    }
  } else {
    // -------------------------------------------------------------- softmax warpgroups
    setmaxnreg_inc<kFaRegsSoftmax>();
    const int t = warp >> 2;
    const int lg = warp & 3;  // TMEM lane quarter this warp may access
    const int r = lg * 32 + lane;
    const int row = q0 + t * kFaRows + r;
    const uint32_t lane_off = (uint32_t)(lg * 32) << 16;
    const uint32_t tS = tmem + lane_off + kFaColS + t * kFaKeys;
    const uint32_t tO = tmem + lane_off + kFaColO + t * kFaDh;
    const uint32_t tP = tmem + lane_off + kFaColP + t * (kFaKeys / 2);
    const float sl2 = p.scale_log2;
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    int n = nkt[0];
#pragma unroll
    for (int u = 1; u < kFaQTiles; ++u)
      if (t == u) n = nkt[u];  // register select, no local-memory indexing
    for (int j = 0; j < n; ++j) {
      ok = __all_sync(0xffffffffu, mbar_wait(&bar[kFaBarSF + t], j & 1, p.err, 14));
      if (!ok) break;
      tc_fence_after();
      float s[kFaKeys];
#pragma unroll
      for (int c = 0; c < kFaKeys; c += 32) tmem_ld32(tS + c, s + c);
      tmem_ld_wait();
      // S_t is in registers: the MMA thread may overwrite it with the next key tile
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar[kFaBarSE + t]);
      const int key0 = j * kFaKeys;
      if (key0 + kFaKeys > p.nk || (p.causal && key0 + kFaKeys - 1 > q0 + t * kFaRows)) {
        const int lim = p.causal ? min(p.nk, row + 1) : p.nk;  // keys < lim are visible
#pragma unroll
        for (int c = 0; c < kFaKeys; ++c)
          if (key0 + c >= lim) s[c] = -INFINITY;
      }
      // row max: four independent chains of three-input max
      float mx[4];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        mx[c] = s[32 * c];
#pragma unroll
        for (int i = 1; i < 31; i += 2) mx[c] = fmax3(mx[c], s[32 * c + i], s[32 * c + i + 1]);
        mx[c] = fmaxf(mx[c], s[32 * c + 31]);
      }
      const float m_new = fmaxf(m_used, fmax3(mx[0], mx[1], fmaxf(mx[2], mx[3])) * sl2);
      const bool need = m_new > m_used + 8.f;
      const float fac = need ? ex2_approx(m_used - m_new) : 1.f;
      if (need) {
        l *= fac;
        m_used = m_new;
      }
      const float mb = m_used == -INFINITY ? 0.f : m_used;
      if (j > 0) {
        // P V of the previous key tile has finished: P_t is free and O_t is stable
        ok = __all_sync(0xffffffffu, mbar_wait(&bar[kFaBarOF + t], (j - 1) & 1, p.err, 15));
        if (!ok) break;
        tc_fence_after();
        if (__any_sync(0xffffffffu, need)) {
#pragma unroll
          for (int c = 0; c < kFaDh; c += 16) {
            float o[16];
            tmem_ld16(tO + c, o);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 16; ++i) o[i] *= fac;
            tmem_st16(tO + c, o);
          }
        }
      }
      // p = 2^(s*scale*log2e - m) as bf16 pairs into P_t, 64 keys (32 columns) at a time;
      // scale-subtract and row sums on packed fp32 pairs, four partial sums
      const float2 sl2v = make_float2(sl2, sl2), nmb = make_float2(-mb, -mb);
      float2 acc[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
      for (int h = 0; h < kFaKeys; h += 64) {
        uint32_t pk[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float2 x = fma2(make_float2(s[h + 2 * i], s[h + 2 * i + 1]), sl2v, nmb);
          const float2 e = make_float2(ex2_approx(x.x), ex2_approx(x.y));
          acc[i & 3] = add2(acc[i & 3], e);
          pk[i] = pack_bf16x2(e.x, e.y);
        }
        tmem_st32(tP + h / 2, pk);
      }
      const float2 a01 = add2(acc[0], acc[1]), a23 = add2(acc[2], acc[3]);
      l += (a01.x + a23.x) + (a01.y + a23.y);
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar[kFaBarPF + t]);
    }
    if (ok && n > 0) {
      ok = __all_sync(0xffffffffu, mbar_wait(&bar[kFaBarOF + t], (n - 1) & 1, p.err, 16));
      if (ok) {
        tc_fence_after();
        float o[kFaDh];
#pragma unroll
        for (int c = 0; c < kFaDh; c += 16) tmem_ld16(tO + c, o + c);
        tmem_ld_wait();
        const float inv = 1.f / l;
#pragma unroll
        for (int i = 0; i < kFaDh; ++i) o[i] *= inv;
        if (row < p.nq) {
          __nv_bfloat16* dst = p.out + ((size_t)bh * p.nq + row) * kFaDh;
#pragma unroll
          for (int c = 0; c < kFaDh; c += 8) store8(dst + c, o + c);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kFaMmaWarp) tmem_dealloc(tmem, kFaTmemCols);
}

// x * cos + rotate_half(x) * sin (one/flash_attention.py:20-33) on q and k rows of 64,
// each product and the sum rounded to bf16 like the reference's elementwise ops. One
// thread per 8-element chunk of the first half and the matching chunk of the second.
// cos / sin are [B, n, 64] with batch stride `cs_bstride` elements (0: shared).
__global__ void rope_qk_kernel(const __nv_bfloat16* q, const __nv_bfloat16* k, const __nv_bfloat16* cosv,
                               const __nv_bfloat16* sinv, int h, int n, long cs_bstride, long rows,
                               __nv_bfloat16* qr, __nv_bfloat16* kr) {
  pdl_wait();
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows * 8) return;
  const int c = (int)(i & 3) * 8;
  long row = i >> 2;
  const bool is_k = row >= rows;
  if (is_k) row -= rows;
  const long bhi = row / n;
  const int pos = (int)(row - bhi * n);
  const long b = bhi / h;
  const __nv_bfloat16* x = (is_k ? k : q) + row * 64;
  const __nv_bfloat16* cs = cosv + b * cs_bstride + (long)pos * 64;
  const __nv_bfloat16* sn = sinv + b * cs_bstride + (long)pos * 64;
  float x1[8], x2[8], c1[8], c2[8], s1[8], s2[8], o1[8], o2[8];
  load8(x + c, x1);
  load8(x + 32 + c, x2);
  load8(cs + c, c1);
  load8(cs + 32 + c, c2);
  load8(sn + c, s1);
  load8(sn + 32 + c, s2);
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    o1[e] = rnd<__nv_bfloat16>(x1[e] * c1[e]) + rnd<__nv_bfloat16>(-x2[e] * s1[e]);
    o2[e] = rnd<__nv_bfloat16>(x2[e] * c2[e]) + rnd<__nv_bfloat16>(x1[e] * s2[e]);
  }
  __nv_bfloat16* y = (is_k ? kr : qr) + row * 64;
  store8(y + c, o1);
  store8(y + 32 + c, o2);
}

}  // namespace one
