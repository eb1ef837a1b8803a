// Token sampling for generate(do_sample=True): per sequence, the logits warped as the HF
// generation loop warps them (transformers generation/utils.py _get_logits_processor, sampling
// branch, in this order: TemperatureLogitsWarper scores / T, TopKLogitsWarper (keep scores >=
// the k-th largest), TopPLogitsWarper (keep the largest tokens until their probability mass
// reaches top_p, at least one)), then one multinomial draw from softmax of the kept scores.
//
// One CTA of kSampThreads threads per sequence, the warped scores in shared memory. The k-th
// largest score and the top-p boundary are found by
// radix selection over order-preserving 32-bit keys of the fp32 scores (4 rounds of 8 bits):
// counts for top-k, and for top-p masses in 2^-32 fixed point (integer atomics: the boundary
// does not depend on the order of the additions, so a seed always draws the same tokens).
// Ties at a boundary are all kept (HF's sort order among equal scores is unspecified).
// The uniform variate comes from Philox4x32-10 (Salmon, Moraes, Dror, Shaw: "Parallel random
// numbers: as easy as 1, 2, 3", SC 2011) keyed by the seed, counter (offset, sequence).
#pragma once

#include "common.cuh"

namespace one {

constexpr int kSampThreads = 1024;
constexpr int kSampMaxVocab = 49152;  // fp32 scores held in shared memory (192 KB)

struct SampleParams {
  const void* logits;  // [batch][ld], model dtype
  int batch, vocab, ld, dtype;
  float temperature;   // > 0
  int top_k;           // 0: off
  float top_p;         // >= 1: off
  unsigned long long seed, offset;
  int* out;            // [batch]
};

ONE_DEVINL uint32_t f32_key(float f) {
  const uint32_t b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// Philox4x32 with 10 rounds; returns the first output word.
ONE_DEVINL uint32_t philox4x32_10(uint32_t c0, uint32_t c1, uint32_t c2, uint32_t c3, uint32_t k0, uint32_t k1) {
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint32_t hi0 = __umulhi(0xD2511F53u, c0), lo0 = 0xD2511F53u * c0;
    const uint32_t hi1 = __umulhi(0xCD9E8D57u, c2), lo1 = 0xCD9E8D57u * c2;
    const uint32_t n0 = hi1 ^ c1 ^ k0, n1 = lo1, n2 = hi0 ^ c3 ^ k1, n3 = lo0;
    c0 = n0; c1 = n1; c2 = n2; c3 = n3;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  return c0;
}

struct SampShared {
  unsigned long long hist[256];
  unsigned long long red[kSampThreads / 32];
  float redf[kSampThreads / 32];
  unsigned long long sel_mass;
  uint32_t sel_digit;
  int pick;
};

// Weight of a kept score for the top-p and sampling passes: exp(s - mx) in 2^-32 fixed point,
// at least 1 (a kept token keeps a nonzero chance).
ONE_DEVINL unsigned long long samp_weight(float s, float mx) {
  const unsigned long long w = (unsigned long long)(expf(s - mx) * 4294967296.0f);
  return w ? w : 1ull;
}

// Radix selection over the scores whose key is >= `floor`: the largest key K such that the
// weight (1 per entry when `mass` is false, samp_weight otherwise) of the entries with key >= K
// reaches `need`. Four rounds of 8-bit digits from the top.
ONE_DEVINL uint32_t radix_boundary(const float* sc, int V, uint32_t floor, bool mass, float mx, unsigned long long need,
                                   SampShared& sh) {
  uint32_t prefix = 0, mask = 0;
  unsigned long long above = 0;  // weight of entries above the current prefix
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = threadIdx.x; i < 256; i += blockDim.x) sh.hist[i] = 0ull;
    __syncthreads();
    for (int v = threadIdx.x; v < V; v += blockDim.x) {
      const float x = sc[v];
      const uint32_t k = f32_key(x);
      if (k >= floor && (k & mask) == prefix) atomicAdd(&sh.hist[(k >> shift) & 0xFFu], mass ? samp_weight(x, mx) : 1ull);
    }
    __syncthreads();
    if (threadIdx.x < 32) {
      // lane l sums digits 255 - 8l .. 248 - 8l; the first digit (from the top) where the
      // running weight reaches `need` is selected
      const int lane = threadIdx.x;
      unsigned long long part = 0;
      for (int d = 255 - 8 * lane; d > 247 - 8 * lane; --d) part += sh.hist[d];
      unsigned long long incl = part;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const unsigned long long t = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += t;
      }
      const unsigned long long excl = incl - part;
      const unsigned ball = __ballot_sync(0xffffffffu, above + incl >= need);
      const int src = ball ? __ffs(ball) - 1 : 31;
      if (lane == src) {
        unsigned long long acc = above + excl;
        int dsel = 248 - 8 * lane;
        for (int d = 255 - 8 * lane; d > 247 - 8 * lane; --d) {
          if (acc + sh.hist[d] >= need) {
            dsel = d;
            break;
          }
          acc += sh.hist[d];
        }
        sh.sel_digit = (uint32_t)dsel;
        sh.sel_mass = acc;
      }
    }
    __syncthreads();
    prefix |= sh.sel_digit << shift;
    mask |= 0xFFu << shift;
    above = sh.sel_mass;
    __syncthreads();
  }
  return prefix;
}

ONE_DEVINL unsigned long long samp_block_sum(unsigned long long v, SampShared& sh) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  if (lane == 0) sh.red[warp] = v;
  __syncthreads();
  unsigned long long t = 0;
  for (int i = 0; i < kSampThreads / 32; ++i) t += sh.red[i];
  return t;
}

__global__ void __launch_bounds__(kSampThreads, 1) sample_kernel(const SampleParams p) {
  extern __shared__ float sc[];  // [vocab] warped scores
  __shared__ SampShared sh;
  pdl_wait();
  const int row = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int V = p.vocab;
  // ---- scores / T in fp32, as HF warps the fp32 logits; NaN scores are never drawn
  float mx = -INFINITY;
  for (int v = tid; v < V; v += blockDim.x) {
    float x = p.dtype == ONE_DTYPE_BF16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p.logits)[(size_t)row * p.ld + v])
                                        : reinterpret_cast<const float*>(p.logits)[(size_t)row * p.ld + v];
    x = x / p.temperature;
    if (isnan(x)) x = -INFINITY;
    sc[v] = x;
  }
  __syncthreads();
  // ---- top-k (TopKLogitsWarper): keep scores >= the k-th largest
  uint32_t floor = 0u;
  if (p.top_k > 0 && p.top_k < V) floor = radix_boundary(sc, V, 0u, false, 0.f, (unsigned long long)p.top_k, sh);
  // ---- softmax weights of the kept scores
  for (int v = tid; v < V; v += blockDim.x)
    if (f32_key(sc[v]) >= floor) mx = fmaxf(mx, sc[v]);
  mx = warp_max(mx);
  if (lane == 0) sh.redf[warp] = mx;
  __syncthreads();
  mx = sh.redf[0];
  for (int i = 1; i < kSampThreads / 32; ++i) mx = fmaxf(mx, sh.redf[i]);
  __syncthreads();
  const bool any = mx > -INFINITY;
  // ---- top-p (TopPLogitsWarper): keep the largest tokens until their mass reaches top_p
  if (any && p.top_p < 1.0f) {
    unsigned long long z = 0;
    for (int v = tid; v < V; v += blockDim.x)
      if (f32_key(sc[v]) >= floor) z += samp_weight(sc[v], mx);
    const unsigned long long Z = samp_block_sum(z, sh);
    const double need_d = (double)fmaxf(p.top_p, 0.f) * (double)Z;
    unsigned long long need = (unsigned long long)need_d;
    if ((double)need < need_d) ++need;
    if (need < 1) need = 1;
    floor = radix_boundary(sc, V, floor, true, mx, need, sh);
  }
  // ---- one multinomial draw: the first token in vocabulary order whose inclusive prefix weight
  //      exceeds u * Z. Thread t takes the contiguous entries [t * per, (t + 1) * per).
  const int per = (V + kSampThreads - 1) / kSampThreads;
  const int v0 = tid * per, v1 = min(V, v0 + per);
  unsigned long long mine = 0;
  if (any)
    for (int v = v0; v < v1; ++v)
      if (f32_key(sc[v]) >= floor) mine += samp_weight(sc[v], mx);
  unsigned long long incl = mine;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned long long t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  __syncthreads();
  if (lane == 31) sh.red[warp] = incl;
  if (tid == 0) sh.pick = -1;
  __syncthreads();
  unsigned long long Z = 0, wbase = 0;
  for (int i = 0; i < kSampThreads / 32; ++i) {
    if (i < warp) wbase += sh.red[i];
    Z += sh.red[i];
  }
  const uint32_t r = philox4x32_10((uint32_t)p.offset, (uint32_t)(p.offset >> 32), (uint32_t)row, 0u,
                                   (uint32_t)p.seed, (uint32_t)(p.seed >> 32));
  const double u = (double)(r >> 8) * (1.0 / 16777216.0);  // [0, 1), 24 bits
  const unsigned long long target = (unsigned long long)(u * (double)Z);
  unsigned long long acc = wbase + incl - mine;
  if (Z > 0 && acc <= target && target < acc + mine) {
    for (int v = v0; v < v1; ++v) {
      if (f32_key(sc[v]) < floor) continue;
      const unsigned long long w = samp_weight(sc[v], mx);
      if (target < acc + w) {
        sh.pick = v;
        break;
      }
      acc += w;
    }
  }
  __syncthreads();
  if (tid == 0) p.out[row] = sh.pick >= 0 ? sh.pick : 0;  // no finite score: token 0
}

}  // namespace one
