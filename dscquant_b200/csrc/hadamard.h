// Host-side constructions of +-1 Hadamard matrices used by the Kronecker
// rotations H_a (x) H_b (the reference has no online rotation; these are
// built from the mathematics):
//   * Sylvester:  order 2^j, H[r][c] = (-1)^popcount(r & c)
//   * Paley I:    order q+1 for a prime q = 3 (mod 4)
//   * Paley II:   order 2(q+1) for a prime q = 1 (mod 4)   (28 = 2*(13+1))
//   * Goethals-Seidel array over four circulant +-1 matrices of order 43
//     whose sequences are constant on the cosets of the order-7 subgroup of
//     Z_43^* (primitive root 3); the four coset patterns below give
//     A A^T + B B^T + C C^T + D D^T = 172 I, hence a Hadamard matrix of order
//     172 (= 4*43). The patterns were found by an exhaustive search over the
//     2^7 coset-constant sequences (meet in the middle on periodic
//     autocorrelations); oracle/hadamard_search.c reproduces it.
#pragma once
#include <stdint.h>
#include <string.h>
#include <vector>

namespace dscq {

inline bool is_prime(int q) {
  if (q < 2) return false;
  for (int d = 2; d * d <= q; ++d)
    if (q % d == 0) return false;
  return true;
}

inline int legendre(int x, int q) {  // quadratic character of x mod prime q
  x %= q;
  if (x < 0) x += q;
  if (x == 0) return 0;
  int r = 1, b = x, e = (q - 1) / 2;
  while (e) {
    if (e & 1) r = static_cast<int>(static_cast<int64_t>(r) * b % q);
    b = static_cast<int>(static_cast<int64_t>(b) * b % q);
    e >>= 1;
  }
  return r == 1 ? 1 : -1;
}

// Writes a +-1 Hadamard matrix of order n (row-major) into h; returns false if
// no construction here covers n.
inline bool build_hadamard(int n, int8_t* h) {
  if (n < 1) return false;
  if ((n & (n - 1)) == 0) {
    for (int r = 0; r < n; ++r)
      for (int c = 0; c < n; ++c) h[r * n + c] = (__builtin_popcount(r & c) & 1) ? -1 : 1;
    return true;
  }
  if (n == 172) {
    const int m = 43, e = 6, g = 3;
    const uint32_t pattern[4] = {14u, 26u, 38u, 60u};  // bit0: value at 0; bit 1+c: value on coset c
    int coset[43];
    for (int k = 0, v = 1; k < m - 1; ++k, v = v * g % m) coset[v] = k % e;
    int seq[4][43];
    for (int s = 0; s < 4; ++s) {
      seq[s][0] = (pattern[s] & 1u) ? -1 : 1;
      for (int x = 1; x < m; ++x) seq[s][x] = ((pattern[s] >> (1 + coset[x])) & 1u) ? -1 : 1;
    }
    // circulant X[i][j] = x[(j - i) mod m]; R = back-diagonal permutation
    auto C = [&](int s, int i, int j) { return seq[s][((j - i) % m + m) % m]; };
    auto CR = [&](int s, int i, int j) { return C(s, i, m - 1 - j); };   // X R
    auto CtR = [&](int s, int i, int j) { return C(s, m - 1 - j, i); };  // X^T R
    // Goethals-Seidel array
    // [  A    BR    CR    DR  ]
    // [ -BR   A     D^TR -C^TR]
    // [ -CR  -D^TR  A     B^TR]
    // [ -DR   C^TR -B^TR  A   ]
    for (int bi = 0; bi < 4; ++bi)
      for (int bj = 0; bj < 4; ++bj)
        for (int i = 0; i < m; ++i)
          for (int j = 0; j < m; ++j) {
            int v = 0;
            const int A = 0, B = 1, Cc = 2, D = 3;
            switch (bi * 4 + bj) {
              case 0: v = C(A, i, j); break;
              case 1: v = CR(B, i, j); break;
              case 2: v = CR(Cc, i, j); break;
              case 3: v = CR(D, i, j); break;
              case 4: v = -CR(B, i, j); break;
              case 5: v = C(A, i, j); break;
              case 6: v = CtR(D, i, j); break;
              case 7: v = -CtR(Cc, i, j); break;
              case 8: v = -CR(Cc, i, j); break;
              case 9: v = -CtR(D, i, j); break;
              case 10: v = C(A, i, j); break;
              case 11: v = CtR(B, i, j); break;
              case 12: v = -CR(D, i, j); break;
              case 13: v = CtR(Cc, i, j); break;
              case 14: v = -CtR(B, i, j); break;
              case 15: v = C(A, i, j); break;
            }
            h[(bi * m + i) * n + bj * m + j] = static_cast<int8_t>(v);
          }
    return true;
  }
  if (n % 4 == 0 && is_prime(n - 1) && (n - 1) % 4 == 3) {
    // Paley I: H = I + S with S = [[0, 1^T], [-1, Q]], Q[i][j] = chi(j - i)
    const int q = n - 1;
    for (int r = 0; r < n; ++r)
      for (int c = 0; c < n; ++c) {
        int s;
        if (r == 0 && c == 0) s = 0;
        else if (r == 0) s = 1;
        else if (c == 0) s = -1;
        else s = legendre((c - 1) - (r - 1), q);
        h[r * n + c] = static_cast<int8_t>(s + (r == c ? 1 : 0));
      }
    return true;
  }
  if (n % 4 == 0 && is_prime(n / 2 - 1) && (n / 2 - 1) % 4 == 1) {
    // Paley II: conference matrix C = [[0, 1^T], [1, Q]] (symmetric),
    // H = C (x) [[1, 1], [1, -1]] + I (x) [[1, -1], [-1, -1]]
    const int q = n / 2 - 1, m = q + 1;
    for (int r = 0; r < m; ++r)
      for (int c = 0; c < m; ++c) {
        int cv;
        if (r == 0 && c == 0) cv = 0;
        else if (r == 0 || c == 0) cv = 1;
        else cv = legendre((c - 1) - (r - 1), q);
        const int e = (r == c) ? 1 : 0;
        const int blk1[2][2] = {{1, 1}, {1, -1}}, blk2[2][2] = {{1, -1}, {-1, -1}};
        for (int u = 0; u < 2; ++u)
          for (int v = 0; v < 2; ++v) h[(2 * r + u) * n + 2 * c + v] = static_cast<int8_t>(cv * blk1[u][v] + e * blk2[u][v]);
      }
    return true;
  }
  return false;
}

// Splits K = a * 2^j with a the dense factor used for the online rotation:
// 1 for powers of two, otherwise 4 * (odd part of K) when a Hadamard matrix of
// that order is constructible here (11008 -> 172 x 64, 14336 -> 28 x 512,
// 28672 -> 28 x 1024). Returns false if K has no supported split.
inline bool rotation_split(int64_t K, int* a_out, int* log2b_out) {
  if (K < 1) return false;
  int64_t odd = K;
  int j = 0;
  while ((odd & 1) == 0) {
    odd >>= 1;
    ++j;
  }
  if (odd == 1) {
    *a_out = 1;
    *log2b_out = j;
    return true;
  }
  if (j < 2 || odd > 1024) return false;
  const int a = static_cast<int>(4 * odd);
  std::vector<int8_t> tmp(static_cast<size_t>(a) * a);
  if (!build_hadamard(a, tmp.data())) return false;
  *a_out = a;
  *log2b_out = j - 2;
  return true;
}

}  // namespace dscq
