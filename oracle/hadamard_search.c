// ORACLE / test infrastructure: reproduces the coset patterns behind the
// order-172 Hadamard matrix of dscquant_b200/csrc/hadamard.h.
//
// Searches four +-1 sequences of length 43, each constant on the cosets of a
// subgroup H (|H| = h) of Z_43^*, whose periodic autocorrelations sum to zero
// at every nonzero shift. Their circulants in the Goethals-Seidel array give a
// Hadamard matrix of order 172. Sequences are grouped by row sum (the four
// row sums r_i satisfy sum r_i^2 = 172) and paired by a meet-in-the-middle
// hash on autocorrelation vectors (constant on cosets, so e = 42/h values).
// Usage: hadamard_search <h>     (h = 7 prints the patterns 14 26 38 60)
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <stdint.h>
#define N 43
static int prim, h, e, coset_of[N];
static int seq_from_bits(uint32_t bits, int8_t *a) {
  a[0] = (bits & 1) ? -1 : 1; int s = a[0];
  for (int x = 1; x < N; x++) { a[x] = (bits >> (1 + coset_of[x])) & 1 ? -1 : 1; s += a[x]; }
  return s;
}
static void paf(const int8_t *a, int16_t *v) { // one value per coset (shift representative)
  int rep[64]; for (int c = 0; c < e; c++) rep[c] = -1;
  for (int x = 1; x < N; x++) if (rep[coset_of[x]] < 0) rep[coset_of[x]] = x;
  for (int c = 0; c < e; c++) { int s = rep[c], t = 0; for (int x = 0; x < N; x++) t += a[x] * a[(x + s) % N]; v[c] = t; }
}
typedef struct { uint64_t key; uint32_t i, j; } Ent;
static uint64_t hv(const int16_t *v) { uint64_t k = 1469598103934665603ull; for (int c = 0; c < e; c++) { k ^= (uint16_t)v[c]; k *= 1099511628211ull; } return k; }
static int cmp(const void *x, const void *y) { uint64_t a = ((Ent*)x)->key, b = ((Ent*)y)->key; return a < b ? -1 : a > b; }
int main(int argc, char **argv) {
  h = atoi(argv[1]);
  for (prim = 2; prim < N; prim++) { int o = 1, v = prim; while (v != 1) { v = v * prim % N; o++; } if (o == N - 1) break; }
  e = (N - 1) / h;
  // coset index of g^k is k mod e
  int v = 1; for (int k = 0; k < N - 1; k++) { coset_of[v] = k % e; v = v * prim % N; }
  int nb = 1 + e; uint32_t total = 1u << nb;
  fprintf(stderr, "prim=%d h=%d e=%d sequences=%u\n", prim, h, e, total);
  int8_t a[N]; int16_t *P = malloc(sizeof(int16_t) * e * (total / 2)); int *S = malloc(sizeof(int) * (total / 2));
  uint32_t cnt = 0; // a0 = +1 (bit0 = 0), sign of whole sequence free
  for (uint32_t b = 0; b < total; b += 2) { S[cnt] = seq_from_bits(b, a); paf(a, P + (size_t)cnt * e); cnt++; }
  int decs[8][4], nd = 0;
  for (int r1 = 1; r1 < 14; r1 += 2) for (int r2 = r1; r2 < 14; r2 += 2) for (int r3 = r2; r3 < 14; r3 += 2) for (int r4 = r3; r4 < 14; r4 += 2)
    if (r1*r1 + r2*r2 + r3*r3 + r4*r4 == 4 * N) { decs[nd][0]=r1; decs[nd][1]=r2; decs[nd][2]=r3; decs[nd][3]=r4; nd++; }
  for (int d = 0; d < nd; d++) {
    int *r = decs[d];
    // lists by |sum|
    uint32_t *L[4]; uint32_t n[4];
    for (int q = 0; q < 4; q++) { L[q] = malloc(sizeof(uint32_t) * cnt); n[q] = 0; for (uint32_t i = 0; i < cnt; i++) if (abs(S[i]) == r[q]) L[q][n[q]++] = i; }
    fprintf(stderr, "dec %d %d %d %d: sizes %u %u %u %u\n", r[0], r[1], r[2], r[3], n[0], n[1], n[2], n[3]);
    if (!n[0] || !n[1] || !n[2] || !n[3]) continue;
    size_t m = (size_t)n[2] * n[3]; Ent *T = malloc(sizeof(Ent) * m); size_t t = 0; int16_t w[64];
    for (uint32_t i = 0; i < n[2]; i++) for (uint32_t j = 0; j < n[3]; j++) {
      const int16_t *p = P + (size_t)L[2][i] * e, *q = P + (size_t)L[3][j] * e;
      for (int c = 0; c < e; c++) w[c] = -(p[c] + q[c]);
      T[t].key = hv(w); T[t].i = L[2][i]; T[t].j = L[3][j]; t++;
    }
    qsort(T, t, sizeof(Ent), cmp);
    for (uint32_t i = 0; i < n[0]; i++) for (uint32_t j = 0; j < n[1]; j++) {
      const int16_t *p = P + (size_t)L[0][i] * e, *q = P + (size_t)L[1][j] * e;
      for (int c = 0; c < e; c++) w[c] = p[c] + q[c];
      uint64_t k = hv(w); size_t lo = 0, hi = t;
      while (lo < hi) { size_t mid = (lo + hi) / 2; if (T[mid].key < k) lo = mid + 1; else hi = mid; }
      for (; lo < t && T[lo].key == k; lo++) {
        const int16_t *x = P + (size_t)T[lo].i * e, *y = P + (size_t)T[lo].j * e; int ok = 1;
        for (int c = 0; c < e; c++) if (p[c] + q[c] + x[c] + y[c]) { ok = 0; break; }
        if (ok) { printf("FOUND h=%d prim=%d bits %u %u %u %u\n", h, prim, L[0][i] * 2, L[1][j] * 2, T[lo].i * 2, T[lo].j * 2); fflush(stdout); return 0; }
      }
    }
    free(T); for (int q = 0; q < 4; q++) free(L[q]);
  }
  printf("none for h=%d\n", h); return 1;
}
