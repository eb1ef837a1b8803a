// Router expert selection, step for step the CPU selection torch.topk(..., sorted=False)
// performs (one/linear_moe.py:83-84): a queue of (score, index) pairs reordered by
// libstdc++ std::nth_element (introselect: median-of-3 pivot, unguarded partition,
// insertion sort below 4 elements, heap select at depth 0) when k * 64 > n, and by
// std::partial_sort (heap select + sort_heap) otherwise, with a comparator that looks
// at scores only ("a before b" iff a is NaN and b is not, or a > b). The first k queue
// entries, in queue order, are the chosen experts. Runs in one thread, n <= kMaxExperts.
#pragma once

#include "common.cuh"

namespace one {

#define ONE_HDINL __host__ __device__ __forceinline__

constexpr int kMaxExperts = 64;

// Queue in (local) memory: any n <= kMaxExperts.
struct TopkMemQ {
  float v[kMaxExperts];
  int i[kMaxExperts];
  ONE_HDINL float gv(int j) const { return v[j]; }
  ONE_HDINL int gi(int j) const { return i[j]; }
  ONE_HDINL void set(int j, float x, int ix) { v[j] = x; i[j] = ix; }
};
// Queue in registers for n <= N: every access is an unrolled select over N slots.
template <int N>
struct TopkRegQ {
  float v[N];
  int i[N];
  ONE_HDINL float gv(int j) const {
    float r = v[0];
#pragma unroll
    for (int k = 1; k < N; ++k) r = (j == k) ? v[k] : r;
    return r;
  }
  ONE_HDINL int gi(int j) const {
    int r = i[0];
#pragma unroll
    for (int k = 1; k < N; ++k) r = (j == k) ? i[k] : r;
    return r;
  }
  ONE_HDINL void set(int j, float x, int ix) {
#pragma unroll
    for (int k = 0; k < N; ++k)
      if (j == k) { v[k] = x; i[k] = ix; }
  }
};

ONE_HDINL bool tk_gt(float a, float b) {
  const bool an = isnan(a), bn = isnan(b);
  return (an && !bn) || (a > b);
}
template <class Q>
ONE_HDINL void tk_swap(Q& q, int a, int b) {
  const float va = q.gv(a), vb = q.gv(b);
  const int ia = q.gi(a), ib = q.gi(b);
  q.set(a, vb, ib);
  q.set(b, va, ia);
}
template <class Q>
ONE_HDINL void tk_insertion_sort(Q& q, int lo, int hi) {
  for (int i = lo + 1; i < hi; ++i) {
    const float v = q.gv(i);
    const int ix = q.gi(i);
    if (tk_gt(v, q.gv(lo))) {
      for (int j = i; j > lo; --j) q.set(j, q.gv(j - 1), q.gi(j - 1));
      q.set(lo, v, ix);
    } else {
      int j = i;
      while (tk_gt(v, q.gv(j - 1))) {
        q.set(j, q.gv(j - 1), q.gi(j - 1));
        --j;
      }
      q.set(j, v, ix);
    }
  }
}
template <class Q>
ONE_HDINL void tk_median_to_first(Q& q, int r, int a, int b, int c) {
  if (tk_gt(q.gv(a), q.gv(b))) {
    if (tk_gt(q.gv(b), q.gv(c))) tk_swap(q, r, b);
    else if (tk_gt(q.gv(a), q.gv(c))) tk_swap(q, r, c);
    else tk_swap(q, r, a);
  } else if (tk_gt(q.gv(a), q.gv(c))) tk_swap(q, r, a);
  else if (tk_gt(q.gv(b), q.gv(c))) tk_swap(q, r, c);
  else tk_swap(q, r, b);
}
template <class Q>
ONE_HDINL int tk_partition(Q& q, int first, int last, int pivot) {
  const float pv = q.gv(pivot);  // the pivot slot is outside [first, last): never moved here
  while (true) {
    while (tk_gt(q.gv(first), pv)) ++first;
    --last;
    while (tk_gt(pv, q.gv(last))) --last;
    if (!(first < last)) return first;
    tk_swap(q, first, last);
    ++first;
  }
}
// libstdc++ __adjust_heap followed by __push_heap, on q[first .. first+len)
template <class Q>
ONE_HDINL void tk_adjust_heap(Q& q, int first, int hole, int len, float val, int vix) {
  const int top = hole;
  int second = hole;
  while (second < (len - 1) / 2) {
    second = 2 * (second + 1);
    if (tk_gt(q.gv(first + second), q.gv(first + second - 1))) --second;
    q.set(first + hole, q.gv(first + second), q.gi(first + second));
    hole = second;
  }
  if ((len & 1) == 0 && second == (len - 2) / 2) {
    second = 2 * (second + 1);
    q.set(first + hole, q.gv(first + second - 1), q.gi(first + second - 1));
    hole = second - 1;
  }
  int parent = (hole - 1) / 2;
  while (hole > top && tk_gt(q.gv(first + parent), val)) {
    q.set(first + hole, q.gv(first + parent), q.gi(first + parent));
    hole = parent;
    parent = (hole - 1) / 2;
  }
  q.set(first + hole, val, vix);
}
template <class Q>
ONE_HDINL void tk_heap_select(Q& q, int first, int middle, int last) {
  const int len = middle - first;
  if (len >= 2)
    for (int parent = (len - 2) / 2; parent >= 0; --parent)
      tk_adjust_heap(q, first, parent, len, q.gv(first + parent), q.gi(first + parent));
  for (int i = middle; i < last; ++i)
    if (tk_gt(q.gv(i), q.gv(first))) {
      const float v = q.gv(i);
      const int ix = q.gi(i);
      q.set(i, q.gv(first), q.gi(first));
      tk_adjust_heap(q, first, 0, len, v, ix);
    }
}
template <class Q>
ONE_HDINL void tk_sort_heap(Q& q, int first, int last) {
  while (last - first > 1) {
    --last;
    const float v = q.gv(last);
    const int ix = q.gi(last);
    q.set(last, q.gv(first), q.gi(first));
    tk_adjust_heap(q, first, 0, last - first, v, ix);
  }
}
ONE_HDINL int tk_lg(int n) {
#ifdef __CUDA_ARCH__
  return 31 - __clz(n);
#else
  return 31 - __builtin_clz((unsigned)n);
#endif
}

template <class Q>
ONE_HDINL void topk_run(Q& q, int n, int k, int* out) {
  if (k <= 0) return;
  if (k * 64 <= n) {
    tk_heap_select(q, 0, k, n);
    tk_sort_heap(q, 0, k);
  } else if (k - 1 < n) {
    const int nth = k - 1;
    int first = 0, last = n;
    int depth = 2 * tk_lg(n);
    bool done = false;
    while (last - first > 3) {
      if (depth == 0) {
        tk_heap_select(q, first, nth + 1, last);
        tk_swap(q, first, nth);
        done = true;
        break;
      }
      --depth;
      const int mid = first + (last - first) / 2;
      tk_median_to_first(q, first, first + 1, mid, last - 1);
      const int cut = tk_partition(q, first + 1, last, first);
      if (cut <= nth) first = cut;
      else last = cut;
    }
    if (!done) tk_insertion_sort(q, first, last);
  }
  for (int j = 0; j < k; ++j) out[j] = q.gi(j);
}

// Select k of n scores; writes the chosen indices, in the reference's order, to out[0..k).
ONE_HDINL void topk_select(const float* score, int n, int k, int* out) {
  if (false) {  // the register queue is slower than the local-memory one (measured)
    TopkRegQ<8> q;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      q.v[j] = j < n ? score[j] : 0.f;
      q.i[j] = j;
    }
    topk_run(q, n, k, out);
  } else {
    TopkMemQ q;
    for (int j = 0; j < n; ++j) q.set(j, score[j], j);
    topk_run(q, n, k, out);
  }
}

// The selection topk_select makes on n equal scores, packed one index per byte (k <= 8):
// it depends only on (n, k), so hosts compute it once and pass it to the kernels.
inline unsigned long long topk_tie_selection(int n, int k) {
  n = n < 1 ? 1 : (n > kMaxExperts ? kMaxExperts : n);
  k = k < 1 ? 1 : (k > n ? n : k);
  float z[kMaxExperts];
  int out[kMaxExperts];
  for (int j = 0; j < n; ++j) z[j] = 0.f;
  topk_select(z, n, k, out);
  unsigned long long packed = 0;
  for (int j = 0; j < k && j < 8; ++j) packed |= (unsigned long long)(out[j] & 0xFF) << (8 * j);
  return packed;
}

// topk_select with two exact shortcuts, checked on the scores first (one thread):
//   * every score equal (and not NaN), k <= 8: the selection depends only on (n, k), so the
//     caller passes `tie`, topk_tie_selection(n, k);
//   * k <= 2 and the top k + 1 scores strictly ordered (no NaN): nth_element and
//     partial_sort both place the largest first and, for k = 2, the second largest next.
// Any other pattern (ties among the top k + 1, NaN) runs the full selection.
ONE_DEVINL void topk_select_fast(const float* score, int n, int k, int* out, unsigned long long tie) {
  if (k <= 2 && n >= 1) {
    bool nan = false, all_eq = true;
    float v1 = -INFINITY, v2 = -INFINITY, v3 = -INFINITY;
    int i1 = 0, i2 = 0;
    const float s0 = score[0];
    for (int j = 0; j < n; ++j) {
      const float x = score[j];
      nan |= isnan(x);
      all_eq &= x == s0;
      if (x > v1) {
        v3 = v2;
        v2 = v1;
        i2 = i1;
        v1 = x;
        i1 = j;
      } else if (x > v2) {
        v3 = v2;
        v2 = x;
        i2 = j;
      } else if (x > v3) {
        v3 = x;
      }
    }
    // a score equal to the current first / second never replaces it, so a tie leaves v1 == v2
    // or v2 == v3 behind ("x > v2" admits x == v1 as the new second)
    if (!nan) {
      if (all_eq) {
        for (int j = 0; j < k; ++j) out[j] = (int)((tie >> (8 * j)) & 0xFF);
        return;
      }
      if (k == 1 && n >= 2 && v1 > v2) {
        out[0] = i1;
        return;
      }
      if (k == 2 && n >= 3 && v1 > v2 && v2 > v3) {
        out[0] = i1;
        out[1] = i2;
        return;
      }
    }
  }
  topk_select(score, n, k, out);
}

}  // namespace one
