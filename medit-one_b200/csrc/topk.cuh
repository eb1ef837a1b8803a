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

constexpr int kMaxExperts = 64;

struct TopkQ {
  float v[kMaxExperts];
  int i[kMaxExperts];
};

ONE_DEVINL bool tk_gt(float a, float b) {
  const bool an = isnan(a), bn = isnan(b);
  return (an && !bn) || (a > b);
}
ONE_DEVINL void tk_swap(TopkQ& q, int a, int b) {
  float tv = q.v[a]; q.v[a] = q.v[b]; q.v[b] = tv;
  int ti = q.i[a]; q.i[a] = q.i[b]; q.i[b] = ti;
}
ONE_DEVINL void tk_insertion_sort(TopkQ& q, int lo, int hi) {
  for (int i = lo + 1; i < hi; ++i) {
    const float v = q.v[i];
    const int ix = q.i[i];
    if (tk_gt(v, q.v[lo])) {
      for (int j = i; j > lo; --j) { q.v[j] = q.v[j - 1]; q.i[j] = q.i[j - 1]; }
      q.v[lo] = v; q.i[lo] = ix;
    } else {
      int j = i;
      while (tk_gt(v, q.v[j - 1])) { q.v[j] = q.v[j - 1]; q.i[j] = q.i[j - 1]; --j; }
      q.v[j] = v; q.i[j] = ix;
    }
  }
}
ONE_DEVINL void tk_median_to_first(TopkQ& q, int r, int a, int b, int c) {
  if (tk_gt(q.v[a], q.v[b])) {
    if (tk_gt(q.v[b], q.v[c])) tk_swap(q, r, b);
    else if (tk_gt(q.v[a], q.v[c])) tk_swap(q, r, c);
    else tk_swap(q, r, a);
  } else if (tk_gt(q.v[a], q.v[c])) tk_swap(q, r, a);
  else if (tk_gt(q.v[b], q.v[c])) tk_swap(q, r, c);
  else tk_swap(q, r, b);
}
ONE_DEVINL int tk_partition(TopkQ& q, int first, int last, int pivot) {
  while (true) {
    while (tk_gt(q.v[first], q.v[pivot])) ++first;
    --last;
    while (tk_gt(q.v[pivot], q.v[last])) --last;
    if (!(first < last)) return first;
    tk_swap(q, first, last);
    ++first;
  }
}
// libstdc++ __adjust_heap followed by __push_heap, on q[first .. first+len)
ONE_DEVINL void tk_adjust_heap(TopkQ& q, int first, int hole, int len, float val, int vix) {
  const int top = hole;
  int second = hole;
  while (second < (len - 1) / 2) {
    second = 2 * (second + 1);
    if (tk_gt(q.v[first + second], q.v[first + second - 1])) --second;
    q.v[first + hole] = q.v[first + second]; q.i[first + hole] = q.i[first + second];
    hole = second;
  }
  if ((len & 1) == 0 && second == (len - 2) / 2) {
    second = 2 * (second + 1);
    q.v[first + hole] = q.v[first + second - 1]; q.i[first + hole] = q.i[first + second - 1];
    hole = second - 1;
  }
  int parent = (hole - 1) / 2;
  while (hole > top && tk_gt(q.v[first + parent], val)) {
    q.v[first + hole] = q.v[first + parent]; q.i[first + hole] = q.i[first + parent];
    hole = parent;
    parent = (hole - 1) / 2;
  }
  q.v[first + hole] = val; q.i[first + hole] = vix;
}
ONE_DEVINL void tk_heap_select(TopkQ& q, int first, int middle, int last) {
  const int len = middle - first;
  if (len >= 2)
    for (int parent = (len - 2) / 2;; --parent) {
      tk_adjust_heap(q, first, parent, len, q.v[first + parent], q.i[first + parent]);
      if (parent == 0) break;
    }
  for (int i = middle; i < last; ++i)
    if (tk_gt(q.v[i], q.v[first])) {
      const float v = q.v[i];
      const int ix = q.i[i];
      q.v[i] = q.v[first]; q.i[i] = q.i[first];
      tk_adjust_heap(q, first, 0, len, v, ix);
    }
}
ONE_DEVINL void tk_sort_heap(TopkQ& q, int first, int last) {
  while (last - first > 1) {
    --last;
    const float v = q.v[last];
    const int ix = q.i[last];
    q.v[last] = q.v[first]; q.i[last] = q.i[first];
    tk_adjust_heap(q, first, 0, last - first, v, ix);
  }
}
ONE_DEVINL int tk_lg(int n) { return 31 - __clz(n); }

// Select k of n scores; writes the chosen indices, in the reference's order, to out[0..k).
ONE_DEVINL void topk_select(const float* score, int n, int k, int* out) {
  TopkQ q;
  for (int j = 0; j < n; ++j) { q.v[j] = score[j]; q.i[j] = j; }
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
  for (int j = 0; j < k; ++j) out[j] = q.i[j];
}

}  // namespace one
