// Top-k of a short row in the order torch.topk(largest=True, sorted=True)
// returns it on the CPU, ties included.
//
// The reference ranks split dimensions with CPU torch.topk
// (verify_graph.py:13347 for the input-split driver, :11835-11846 for the
// multi-subbox driver) and the order decides which half each child gets.
// torch fills (score, index) pairs in index order and, with the comparator
// "a before b iff a.score > b.score (NaN first)", runs std::nth_element to
// position k - 1 and std::sort on the first k - 1 pairs when 64 k > n, else
// std::partial_sort (heap selection, then heap sort).  The routines below
// restate those published standard-library algorithms (introselect with a
// median-of-three pivot and an insertion sort below four elements; binary
// heap select / sort) for the array sizes of a branching step.
#pragma once

#include <cuda_runtime.h>

namespace vcb {
namespace {

struct VI {
  float v;
  int i;
};

__device__ __forceinline__ bool tk_before(const VI& a, const VI& b) {
  return (isnan(a.v) && !isnan(b.v)) || a.v > b.v;
}

__device__ void tk_insertion_sort(VI* q, int first, int last) {
  if (first == last) return;
  for (int i = first + 1; i < last; ++i) {
    const VI v = q[i];
    if (tk_before(v, q[first])) {
      for (int j = i; j > first; --j) q[j] = q[j - 1];
      q[first] = v;
    } else {
      int j = i, nxt = i - 1;
      while (tk_before(v, q[nxt])) {
        q[j] = q[nxt];
        j = nxt--;
      }
      q[j] = v;
    }
  }
}

__device__ __forceinline__ void tk_swap(VI* q, int a, int b) {
  const VI t = q[a];
  q[a] = q[b];
  q[b] = t;
}

__device__ void tk_median_to_first(VI* q, int result, int a, int b, int c) {
  if (tk_before(q[a], q[b])) {
    if (tk_before(q[b], q[c])) tk_swap(q, result, b);
    else if (tk_before(q[a], q[c])) tk_swap(q, result, c);
    else tk_swap(q, result, a);
  } else if (tk_before(q[a], q[c])) {
    tk_swap(q, result, a);
  } else if (tk_before(q[b], q[c])) {
    tk_swap(q, result, c);
  } else {
    tk_swap(q, result, b);
  }
}

__device__ int tk_partition(VI* q, int first, int last, int pivot) {
  while (true) {
    while (tk_before(q[first], q[pivot])) ++first;
    --last;
    while (tk_before(q[pivot], q[last])) --last;
    if (!(first < last)) return first;
    tk_swap(q, first, last);
    ++first;
  }
}

__device__ void tk_adjust_heap(VI* q, int first, int hole, int len, VI value) {
  const int top = hole;
  int second = hole;
  while (second < (len - 1) / 2) {
    second = 2 * (second + 1);
    if (tk_before(q[first + second], q[first + second - 1])) --second;
    q[first + hole] = q[first + second];
    hole = second;
  }
  if ((len & 1) == 0 && second == (len - 2) / 2) {
    second = 2 * (second + 1);
    q[first + hole] = q[first + second - 1];
    hole = second - 1;
  }
  int parent = (hole - 1) / 2;
  while (hole > top && tk_before(q[first + parent], value)) {
    q[first + hole] = q[first + parent];
    hole = parent;
    parent = (hole - 1) / 2;
  }
  q[first + hole] = value;
}

__device__ void tk_make_heap(VI* q, int first, int last) {
  const int len = last - first;
  if (len < 2) return;
  for (int parent = (len - 2) / 2;; --parent) {
    tk_adjust_heap(q, first, parent, len, q[first + parent]);
    if (parent == 0) return;
  }
}

// heap of q[first, middle) keeps the best; q[i] (i >= middle) is offered in
// turn (`cand` supplies it, so the caller need not store the whole array)
template <typename F>
__device__ void tk_heap_select(VI* q, int first, int middle, int last, F cand) {
  tk_make_heap(q, first, middle);
  for (int i = middle; i < last; ++i) {
    const VI v = cand(i);
    if (tk_before(v, q[first])) tk_adjust_heap(q, first, 0, middle - first, v);
  }
}

__device__ void tk_sort_heap(VI* q, int first, int last) {
  while (last - first > 1) {
    --last;
    const VI v = q[last];
    q[last] = q[first];
    tk_adjust_heap(q, first, 0, last - first, v);
  }
}

// q[0, n): (score, index) in index order.  On return q[0, k) holds the top
// k in torch's CPU order.  Needs 64 k > n (the nth_element path).
__device__ void tk_nth_path(VI* q, int n, int k) {
  int first = 0, last = n;
  const int nth = k - 1;
  int depth = 2 * (31 - __clz(n));
  bool sorted_tail = false;
  while (last - first > 3) {
    if (depth == 0) {  // introselect's heap fallback
      tk_heap_select(q, first, nth + 1, last, [&](int i) { return q[i]; });
      tk_swap(q, first, nth);
      sorted_tail = true;
      break;
    }
    --depth;
    const int mid = first + (last - first) / 2;
    tk_median_to_first(q, first, first + 1, mid, last - 1);
    const int cut = tk_partition(q, first + 1, last, first);
    if (cut <= nth) first = cut;
    else last = cut;
  }
  if (!sorted_tail) tk_insertion_sort(q, first, last);
  tk_insertion_sort(q, 0, k - 1);  // std::sort of k - 1 <= 16 pairs
}

// q[0, n): (score, index) in index order.  On return q[0, k) holds the top
// k in torch's CPU order, for any 1 <= k <= n.
__device__ void tk_topk(VI* q, int n, int k) {
  if (64 * k > n) {
    tk_nth_path(q, n, k);
    return;
  }
  tk_heap_select(q, 0, k, n, [&](int i) { return q[i]; });
  tk_sort_heap(q, 0, k);
}

}  // namespace
}  // namespace vcb
