// Exact softmax attention on the 5th-generation tensor cores (tcgen05) for head_dim 64 in
// bf16, and the RoPE prologue of the fused RoPE + attention operator.
//
// Semantics: out = softmax(q k^T * scale [+ causal mask]) v with an fp32 softmax, the
// exact attention of turbo_flash_attention's PyTorch path (one/turbo_ops.py:115-143) and of
// flash_attention()'s exact branch (one/flash_attention.py:242-282). The causal mask is
// top-left aligned (torch.triu(..., diagonal=1)): query i sees keys 0..i.
//
// One CTA takes two 128-row query tiles of one (batch, head) and streams the head's keys
// in 128-key tiles:
//   warp 0      TMA producer: Q tiles once, then K and V tiles through a 3-stage ring
//   warp 1      allocates TMEM; one thread issues tcgen05.mma:
//                 S_t = Q_t K_j^T   (M 128, N 128, K 64; both operands K-major in smem)
//                 O_t += P_t V_j    (M 128, N 64, K 128; P K-major, V MN-major)
//   warps 2-9   two softmax warpgroups, one per query tile, one thread per query row:
//                 S row from TMEM -> running max -> p = 2^(s*scale*log2e - m) -> P row
//                 (bf16, 128-byte swizzle) in smem for the P V MMA; row sums in fp32
// TMEM columns: S_0 [0,128), S_1 [128,256), O_0 [256,320), O_1 [320,384) of a 512-column
// allocation. While one warpgroup exponentiates, the tensor core runs the other tile's
// S and the P V products, so the two tiles ping-pong.
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
constexpr int kFaThreads = 64 + 128 * kFaQTiles;
constexpr uint32_t kFaTile = kFaRows * kFaDh * 2;     // one Q, K or V tile: 16 KB
constexpr uint32_t kFaPTile = kFaRows * kFaKeys * 2;  // one P tile: 32 KB (two 64-key halves)
constexpr uint32_t kFaOffQ = 0;
constexpr uint32_t kFaOffK = kFaOffQ + kFaQTiles * kFaTile;
constexpr uint32_t kFaOffV = kFaOffK + kFaStages * kFaTile;
constexpr uint32_t kFaOffP = kFaOffV + kFaStages * kFaTile;
constexpr uint32_t kFaOffBar = kFaOffP + kFaQTiles * kFaPTile;
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
constexpr uint32_t kFaTmemCols = 512;
static_assert(kFaSmem <= 227 * 1024, "attention tile ring exceeds shared memory");
static_assert(kFaOffK % 1024 == 0 && kFaOffV % 1024 == 0 && kFaOffP % 1024 == 0, "swizzled tiles need 1 KB alignment");

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

// Registers are allocated per SM sub-partition (16384 each): ten warps put three on two of
// them, so the bound is 168 registers per thread.
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
  if (warp == 1) {
    tmem_alloc(tmem_slot, kFaTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
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
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------------ MMA issuer
      constexpr uint32_t idesc_s = umma_idesc_bf16(kFaRows, kFaKeys);
      constexpr uint32_t idesc_o = umma_idesc_bf16_bmn(kFaRows, kFaDh);
      bool ok = mbar_wait(&bar[kFaBarQ], 0, p.err, 7);
      tc_fence_after();
      // S_t = Q_t K_j^T (4 MMAs of K 16) and O_t += P_t V_j (8 MMAs of K 16; P halves 16 KB
      // apart, 32 B per 16 keys inside a half; V advances 2 KB per 16 keys)
      auto issue_s = [&](int t, int s) {
        const uint64_t a = umma_desc_sw128(sm + kFaOffQ + t * kFaTile);
        const uint64_t b = umma_desc_sw128(sm + kFaOffK + s * kFaTile);
#pragma unroll
        for (int kk = 0; kk < kFaDh / 16; ++kk)
          umma_bf16(tmem + t * kFaKeys, a + 2 * kk, b + 2 * kk, idesc_s, kk > 0 ? 1u : 0u);
        umma_commit(&bar[kFaBarSF + t]);
      };
      auto issue_pv = [&](int t, int s, bool acc) {
        const uint64_t a = umma_desc_sw128(sm + kFaOffP + t * kFaPTile);
        const uint64_t b = umma_desc_sw128_mn(sm + kFaOffV + s * kFaTile, kFaTile);
#pragma unroll
        for (int kk = 0; kk < kFaKeys / 16; ++kk) {
          const uint64_t ak = a + (uint64_t)((kk >> 2) * (16384 >> 4) + (kk & 3) * 2);
          const uint64_t bk = b + (uint64_t)(kk * (2048 >> 4));
          umma_bf16(tmem + 2 * kFaKeys + t * kFaDh, ak, bk, idesc_o, (acc || kk > 0) ? 1u : 0u);
        }
        umma_commit(&bar[kFaBarOF + t]);
      };
      if (ok && nkt_max > 0 && (ok = mbar_wait(&bar[kFaBarKF], 0, p.err, 8))) {
        tc_fence_after();
#pragma unroll
        for (int t = 0; t < kFaQTiles; ++t)
          if (nkt[t] > 0) issue_s(t, 0);
        umma_commit(&bar[kFaBarKE]);
      }
      // per key tile j, tile by tile: P_t V_j as soon as softmax t has written P_t, then
      // S_t for key tile j + 1 into the buffer softmax t has just read
      for (int j = 0; ok && j < nkt_max; ++j) {
        const int s = j % kFaStages, s1 = (j + 1) % kFaStages;
        bool k_ready = false;
        if (!(ok = mbar_wait(&bar[kFaBarVF + s], (j / kFaStages) & 1, p.err, 9))) break;
#pragma unroll
        for (int t = 0; t < kFaQTiles; ++t) {
          if (j < nkt[t]) {
            if (!(ok = mbar_wait(&bar[kFaBarPF + t], j & 1, p.err, 10))) break;
            tc_fence_after();
            issue_pv(t, s, j > 0);
          }
          if (j + 1 < nkt[t]) {
            if (!k_ready) {
              if (!(ok = mbar_wait(&bar[kFaBarKF + s1], ((j + 1) / kFaStages) & 1, p.err, 11))) break;
              k_ready = true;
            }
            if (!(ok = mbar_wait(&bar[kFaBarSE + t], j & 1, p.err, 12))) break;
            tc_fence_after();
            issue_s(t, s1);
          }
        }
        if (!ok) break;
        umma_commit(&bar[kFaBarVE + s]);
        if (k_ready) umma_commit(&bar[kFaBarKE + s1]);
      }
      // every MMA issued above completes before TMEM is freed
      umma_commit(&bar[kFaBarDone]);
      mbar_wait(&bar[kFaBarDone], 0, p.err, 13);
    }
  } else {
    // -------------------------------------------------------------- softmax warpgroups
    const int t = (warp - 2) >> 2;
    const int lg = warp & 3;  // TMEM lane quarter this warp may access
    const int r = lg * 32 + lane;
    const int row = q0 + t * kFaRows + r;
    const uint32_t lane_off = (uint32_t)(lg * 32) << 16;
    const uint32_t tS = tmem + lane_off + t * kFaKeys;
    const uint32_t tO = tmem + lane_off + 2 * kFaKeys + t * kFaDh;
    uint8_t* prow = sm + kFaOffP + t * kFaPTile + r * 128;
    const int swz = r & 7;
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
      // scores rounded to bf16 as the reference's bf16 matmul rounds them, kept as packed
      // pairs; masked keys become -inf
      const int key0 = j * kFaKeys;
      const bool masked = key0 + kFaKeys > p.nk || (p.causal && key0 + kFaKeys - 1 > q0 + t * kFaRows);
      const int lim = p.causal ? min(p.nk, row + 1) : p.nk;  // keys < lim are visible
      uint32_t sp[kFaKeys / 2];
      float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
      for (int h = 0; h < kFaKeys; h += 32) {
        float v[32];
        tmem_ld32(tS + h, v);
        tmem_ld_wait();
        if (masked) {
#pragma unroll
          for (int c = 0; c < 32; ++c)
            if (key0 + h + c >= lim) v[c] = -INFINITY;
        }
#pragma unroll
        for (int c = 0; c < 32; c += 2) {
          mx0 = fmaxf(mx0, v[c]);
          mx1 = fmaxf(mx1, v[c + 1]);
          sp[(h + c) / 2] = pack_bf16x2(v[c], v[c + 1]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar[kFaBarSE + t]);
      const float m_new = fmaxf(m_used, rnd<__nv_bfloat16>(fmaxf(mx0, mx1)) * sl2);
      const bool need = m_new > m_used + 8.f;
      const float fac = need ? ex2_approx(m_used - m_new) : 1.f;
      if (need) {
        l *= fac;
        m_used = m_new;
      }
      const float mb = m_used == -INFINITY ? 0.f : m_used;
      if (j > 0) {
        // P V of the previous key tile has finished: the P buffer is free and O is stable
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
          tmem_st_wait();
        }
      }
      // p = 2^(s*scale*log2e - m) -> bf16 P row in shared memory, 8 keys (16 B) at a time, in
      // the 128-byte-swizzled K-major layout the MMA reads (two 64-key halves 16 KB apart)
      float l0 = 0.f, l1 = 0.f;
#pragma unroll
      for (int c8 = 0; c8 < kFaKeys / 8; ++c8) {
        uint32_t pk[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const uint32_t w = sp[4 * c8 + i];
          const float p0 = ex2_approx(fmaf(__uint_as_float(w << 16), sl2, -mb));
          const float p1 = ex2_approx(fmaf(__uint_as_float(w & 0xffff0000u), sl2, -mb));
          l0 += p0;
          l1 += p1;
          pk[i] = pack_bf16x2(p0, p1);
        }
        *reinterpret_cast<uint4*>(prow + (c8 >> 3) * 16384 + (((c8 & 7) ^ swz) << 4)) =
            make_uint4(pk[0], pk[1], pk[2], pk[3]);
      }
      l += l0 + l1;
      fence_proxy_async();
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
  if (warp == 1) tmem_dealloc(tmem, kFaTmemCols);
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
