// Compile-time description of an m-truncated edge frame (lmax L, mmax MM).
//
// m-major rows: m = 0 rows for l = 0..L, then for m = 1..MM the +m rows (l = m..L) followed
// by the -m rows (l = m..L).  Row k has degree row_l(k); rows +m and -m of one degree share
// a radial-modulation slot slot(k) (m = 0 rows: slot l; m block: slot base_m + l - m) and are
// partners (pair(k)).  All functions are constexpr so kernels unroll over rows and over the
// 2l+1 coefficients of each row with no runtime predicates.
#pragma once

namespace maloq {

template <int L, int MM>
struct Frame {
  static constexpr int S = (L + 1) * (L + 1);
  static constexpr int M = MM < L ? MM : L;
  __host__ __device__ static constexpr int rows() {
    int r = L + 1;
    for (int m = 1; m <= M; ++m) r += 2 * (L - m + 1);
    return r;
  }
  static constexpr int R = rows();
  __host__ __device__ static constexpr int n_slots() {
    int s = L + 1;
    for (int m = 1; m <= M; ++m) s += L - m + 1;
    return s;
  }
  static constexpr int NS = n_slots();
  // (m, sign, l) of row k
  __host__ __device__ static constexpr int row_l(int k) {
    if (k <= L) return k;
    k -= L + 1;
    for (int m = 1; m <= M; ++m) {
      const int n = L - m + 1;
      if (k < 2 * n) return m + (k % n);
      k -= 2 * n;
    }
    return -1;
  }
  __host__ __device__ static constexpr int slot(int k) {
    if (k <= L) return k;
    int base = L + 1;
    k -= L + 1;
    for (int m = 1; m <= M; ++m) {
      const int n = L - m + 1;
      if (k < 2 * n) return base + (k % n);
      k -= 2 * n;
      base += n;
    }
    return -1;
  }
  __host__ __device__ static constexpr int pair(int k) {
    if (k <= L) return -1;
    int start = L + 1;
    int kk = k - (L + 1);
    for (int m = 1; m <= M; ++m) {
      const int n = L - m + 1;
      if (kk < 2 * n) return kk < n ? start + kk + n : start + kk - n;
      kk -= 2 * n;
      start += 2 * n;
    }
    return -1;
  }
  // true for the row of a pair that carries the pair (+m row) and for m = 0 rows
  __host__ __device__ static constexpr bool leads(int k) { return pair(k) < 0 || pair(k) > k; }
};

}  // namespace maloq
