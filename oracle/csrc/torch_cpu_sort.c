/*
 * Test oracle (see oracle/__init__.py): the element order produced by the
 * reference's `mass.argsort(-1, descending=True)` on the PyTorch CPU build
 * (attention_backends/flex.py:85).  That call is an unstable sort: PyTorch
 * sorts (value, index) pairs with std::sort and a key-only "greater than"
 * comparator, so the order among equal values is whatever libstdc++'s
 * introsort produces.  This file restates that published algorithm
 * (median-of-three quicksort with unguarded Hoare partitions, heapsort when
 * the depth limit 2*floor(log2 n) runs out, final insertion sort with a
 * 16-element threshold) so that tied values land where the reference puts
 * them.  Pinned against torch 2.11 in tests/test_oracle_golden.py.
 */
#include <stdint.h>

typedef struct {
  float v;
  int32_t i;
} pair_t;

enum { kThreshold = 16 };

static int greater(pair_t a, pair_t b) { return a.v > b.v; }

static void swap_at(pair_t* a, long x, long y) {
  pair_t t = a[x];
  a[x] = a[y];
  a[y] = t;
}

static void move_median_to_first(pair_t* a, long result, long x, long y, long z) {
  if (greater(a[x], a[y])) {
    if (greater(a[y], a[z])) swap_at(a, result, y);
    else if (greater(a[x], a[z])) swap_at(a, result, z);
    else swap_at(a, result, x);
  } else if (greater(a[x], a[z])) {
    swap_at(a, result, x);
  } else if (greater(a[y], a[z])) {
    swap_at(a, result, z);
  } else {
    swap_at(a, result, y);
  }
}

static long unguarded_partition(pair_t* a, long first, long last, long pivot) {
  for (;;) {
    while (greater(a[first], a[pivot])) ++first;
    --last;
    while (greater(a[pivot], a[last])) --last;
    if (!(first < last)) return first;
    swap_at(a, first, last);
    ++first;
  }
}

static void adjust_heap(pair_t* a, long first, long hole, long len, pair_t value) {
  const long top = hole;
  long second = hole;
  while (second < (len - 1) / 2) {
    second = 2 * (second + 1);
    if (greater(a[first + second], a[first + second - 1])) --second;
    a[first + hole] = a[first + second];
    hole = second;
  }
  if ((len & 1) == 0 && second == (len - 2) / 2) {
    second = 2 * (second + 1);
    a[first + hole] = a[first + second - 1];
    hole = second - 1;
  }
  long parent = (hole - 1) / 2;
  while (hole > top && greater(a[first + parent], value)) {
    a[first + hole] = a[first + parent];
    hole = parent;
    parent = (hole - 1) / 2;
  }
  a[first + hole] = value;
}

static void heap_sort(pair_t* a, long first, long last) {
  const long len = last - first;
  if (len >= 2) {
    for (long parent = (len - 2) / 2;; --parent) {
      adjust_heap(a, first, parent, len, a[first + parent]);
      if (parent == 0) break;
    }
  }
  while (last - first > 1) {
    --last;
    pair_t value = a[last];
    a[last] = a[first];
    adjust_heap(a, first, 0, last - first, value);
  }
}

static void introsort_loop(pair_t* a, long first, long last, long depth) {
  while (last - first > kThreshold) {
    if (depth == 0) {
      heap_sort(a, first, last);
      return;
    }
    --depth;
    const long mid = first + (last - first) / 2;
    move_median_to_first(a, first, first + 1, mid, last - 1);
    const long cut = unguarded_partition(a, first + 1, last, first);
    introsort_loop(a, cut, last, depth);
    last = cut;
  }
}

static void unguarded_linear_insert(pair_t* a, long last) {
  pair_t val = a[last];
  long next = last - 1;
  while (greater(val, a[next])) {
    a[last] = a[next];
    last = next;
    --next;
  }
  a[last] = val;
}

static void insertion_sort(pair_t* a, long first, long last) {
  if (first == last) return;
  for (long i = first + 1; i != last; ++i) {
    if (greater(a[i], a[first])) {
      pair_t val = a[i];
      for (long j = i; j > first; --j) a[j] = a[j - 1];
      a[first] = val;
    } else {
      unguarded_linear_insert(a, i);
    }
  }
}

static long floor_log2(long n) {
  long k = 0;
  while (n > 1) {
    n >>= 1;
    ++k;
  }
  return k;
}

/* order[r, :] = argsort(values[r, :], descending) in the reference's order. */
void oracle_argsort_desc(const float* values, long rows, long n, int32_t* order, pair_t* scratch) {
  for (long r = 0; r < rows; ++r) {
    pair_t* a = scratch;
    for (long i = 0; i < n; ++i) {
      a[i].v = values[r * n + i];
      a[i].i = (int32_t)i;
    }
    if (n > 0) {
      introsort_loop(a, 0, n, 2 * floor_log2(n));
      if (n > kThreshold) {
        insertion_sort(a, 0, kThreshold);
        for (long i = kThreshold; i < n; ++i) unguarded_linear_insert(a, i);
      } else {
        insertion_sort(a, 0, n);
      }
    }
    for (long i = 0; i < n; ++i) order[r * n + i] = a[i].i;
  }
}
