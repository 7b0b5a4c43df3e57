/*
 * TEST INFRASTRUCTURE ONLY: the CPU oracle of the GGUF MoE block's integer and byte work.
 *
 * A plain-C restatement of the reference's host algorithms for the MoE hot path, used by tests/, by
 * __graft_entry__.smoke() and by bench.py's cpu_baseline leg as the checker. Nothing in the product library links
 * or calls this file. Parity is pinned by tests/test_oracle.py against
 *   - the reference's own compiled moe_host.cpp / dequant.cpp (oracle/_ref, built by oracle/Makefile), and
 *   - golden vectors written by the reference's NumPy oracle (tests/golden/, made by tests/golden/make_golden.py).
 *
 * Reference files (artlite-project/artlite):
 *   csrc/artlite/moe_host.cpp:24-39    row_sum         numpy's pairwise summation order for short rows
 *   csrc/artlite/moe_host.cpp:45-73   route_rows_scalar  top-k by ordered-int keys, weights in double
 *   csrc/artlite/moe_host.cpp:75-90  exp_nonpos      degree-12 Taylor e^x for x <= 0 (the k == 8 softmax path)
 *   csrc/artlite/moe_host.cpp:98-174  route_rows_avx512  which rows take exp_nonpos (k == 8, softmax, no NaN)
 *   csrc/artlite/moe_host.cpp:176-199  route_rows / moe_route  path choice and argument checks
 *   csrc/artlite/moe_host.cpp:201-235  moe_plan        histogram, scan, stable permute, chunk deal, pos
 *   csrc/artlite/dequant.cpp:21-147    per-format block dequant (fp32, no FMA: build with -ffp-contract=off)
 *
 * Every function returns 0 on success or a negative status (the reference throws artlite::Error instead).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ORACLE_OK 0
#define ORACLE_EINVAL -1
#define ORACLE_ECAPACITY -2

/* numpy's pairwise sum of a short row (moe_host.cpp:24-39): plain for n < 8, else 8 accumulators */
static double row_sum(const double* a, int n) {
  if (n < 8) {
    double s = 0;
    for (int i = 0; i < n; i++) s += a[i];
    return s;
  }
  double r[8];
  for (int j = 0; j < 8; j++) r[j] = a[j];
  int i = 8;
  for (; i + 8 <= n; i += 8)
    for (int j = 0; j < 8; j++) r[j] += a[i + j];
  double s = ((r[0] + r[1]) + (r[2] + r[3])) + ((r[4] + r[5]) + (r[6] + r[7]));
  for (; i < n; i++) s += a[i];
  return s;
}

static const double kMinWeightSum = 6.103515625e-5; /* 2^-14 (moe_host.cpp:41) */

/* e^x for x <= 0 as the reference's vector path computes it (moe_host.cpp:75-90): x = n ln2 + r with a two-part
 * ln 2, a degree-12 Taylor polynomial in r by Horner with fused multiply-adds, times 2^n; x clamped at -708. */
static double exp_nonpos(double x) {
  const double log2e = 1.4426950408889634, ln2hi = 6.93147180369123816490e-01, ln2lo = 1.90821492927058770002e-10;
  static const double c[13] = {1.0,           1.0,            1.0 / 2,        1.0 / 6,      1.0 / 24,
                               1.0 / 120,     1.0 / 720,      1.0 / 5040,     1.0 / 40320,  1.0 / 362880,
                               1.0 / 3628800, 1.0 / 39916800, 1.0 / 479001600};
  x = x > -708.0 ? x : -708.0;
  const double n = nearbyint(x * log2e); /* round half to even (default rounding mode) */
  const double r = fma(-n, ln2lo, fma(-n, ln2hi, x));
  double p = c[12];
  for (int i = 11; i >= 0; i--) p = fma(p, r, c[i]);
  const int64_t e = ((int64_t)n + 1023) << 52;
  double s;
  memcpy(&s, &e, 8);
  return p * s;
}

static inline uint32_t f2u(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  return u;
}

/* A logit's ordered key (moe_host.cpp:55-56): (bits(l + 0) flipped to an unsigned order) << 32 | ~id. */
static inline uint64_t route_key(float l, int x) {
  const uint32_t u = f2u(l + 0.0f);
  return (uint64_t)(u ^ ((u >> 31) ? 0xFFFFFFFFu : 0x80000000u)) << 32 | (uint32_t)(~(uint32_t)x);
}

/* The logit of expert x in a token's row (moe_host.cpp:53-55: column x / per_col at its pitch). */
static inline float logit_at(const float* p, int x, int per_col, int64_t pitch) {
  return p[(int64_t)(x / per_col) * pitch + x % per_col];
}

/* moe_route (moe_host.cpp:186-199, rows as route_rows_scalar :45-73 and, for the weights of k == 8 softmax rows
 * without a NaN on the vector path's shapes, exp_nonpos as route_rows_avx512 :199-212). */
int oracle_moe_route(const float* logits, int64_t n, int64_t row, int per_col, int64_t pitch, int E, int k,
                     int sigmoid, int32_t* ids, float* weights) {
  if (k < 1 || k > E || per_col <= 0 || E % per_col) return ORACLE_EINVAL;
  const int vector_shape = k <= 16 && per_col % 16 == 0 && E % per_col == 0 && E <= 512;
  uint64_t* top = (uint64_t*)malloc(sizeof(uint64_t) * (k + 1));
  double* e = (double*)malloc(sizeof(double) * k);
  if (!top || !e) {
    free(top);
    free(e);
    return ORACLE_EINVAL;
  }
  for (int64_t t = 0; t < n; t++) {
    const float* p = logits + t * row;
    int nt = 0, has_nan = 0;
    for (int x = 0; x < E; x++) {
      const float l = logit_at(p, x, per_col, pitch);
      if (l != l) has_nan = 1;
      const uint64_t key = route_key(l, x);
      if (nt == k && key <= top[k - 1]) continue;
      int j = nt < k ? nt++ : k - 1;
      for (; j > 0 && top[j - 1] < key; j--) top[j] = top[j - 1];
      top[j] = key;
    }
    const int32_t first = (int32_t)(~(uint32_t)top[0]);
    /* (the vector path subtracts logits + 0.0f, moe_host.cpp:152: the same differences, -0 and +0 alike) */
    const double l0 = (double)logit_at(p, first, per_col, pitch);
    const int taylor = vector_shape && !has_nan && k == 8 && !sigmoid;
    for (int j = 0; j < k; j++) {
      const int32_t x = (int32_t)(~(uint32_t)top[j]);
      ids[t * k + j] = x;
      const double l = (double)logit_at(p, x, per_col, pitch);
      if (sigmoid)
        e[j] = 1.0 / (1.0 + exp(-l));
      else
        e[j] = taylor ? exp_nonpos(l - l0) : exp(l - l0);
    }
    double s;
    if (taylor)
      s = ((e[0] + e[1]) + (e[2] + e[3])) + ((e[4] + e[5]) + (e[6] + e[7]));
    else {
      s = row_sum(e, k);
      if (sigmoid && s < kMinWeightSum) s = kMinWeightSum; /* std::max(s, 2^-14): a NaN sum stays NaN */
    }
    for (int j = 0; j < k; j++) weights[t * k + j] = (float)(e[j] / s);
  }
  free(top);
  free(e);
  return ORACLE_OK;
}

/* moe_plan (moe_host.cpp:201-235): an expert's (token, slot) pairs in pair order, in chunks of at most `chunk`, dealt
 * to the cols columns in turn; pos[p] = (c cap + kk) chunk + j. Returns ORACLE_EINVAL on an id outside [0, E),
 * ORACLE_ECAPACITY when a column needs more than cap chunks. */
int oracle_moe_plan(const int32_t* ids, int64_t n, int k, int E, int cols, int cap, int chunk, int32_t* experts,
                    int32_t* counts, int32_t* sizes, int32_t* rows, int64_t* pos) {
  const int64_t pairs = n * k;
  int64_t* start = (int64_t*)calloc((size_t)E + 1, sizeof(int64_t));
  int64_t* at = (int64_t*)malloc(sizeof(int64_t) * ((size_t)E + 1));
  int64_t* by = (int64_t*)malloc(sizeof(int64_t) * (size_t)(pairs ? pairs : 1));
  int rc = ORACLE_OK;
  if (!start || !at || !by) {
    rc = ORACLE_EINVAL;
    goto done;
  }
  for (int64_t p = 0; p < pairs; p++) {
    const int32_t x = ids[p];
    if (x < 0 || x >= E) {
      rc = ORACLE_EINVAL;
      goto done;
    }
    start[x + 1]++;
  }
  for (int x = 0; x < E; x++) start[x + 1] += start[x];
  memcpy(at, start, sizeof(int64_t) * (size_t)E);
  for (int64_t p = 0; p < pairs; p++) by[at[ids[p]]++] = p;
  for (int c = 0; c < cols; c++) counts[c] = 0;
  int64_t j = 0;
  for (int x = 0; x < E; x++)
    for (int64_t a = start[x]; a < start[x + 1]; a += chunk) {
      const int64_t b = a + chunk < start[x + 1] ? a + chunk : start[x + 1];
      const int c = (int)(j % cols);
      const int kk = counts[c]++;
      if (kk >= cap) {
        rc = ORACLE_ECAPACITY;
        goto done;
      }
      experts[c * cap + kk] = x;
      sizes[c * cap + kk] = (int32_t)(b - a);
      int32_t* r = rows + ((int64_t)c * cap + kk) * chunk;
      const int64_t base = ((int64_t)c * cap + kk) * chunk;
      for (int64_t i = a; i < b; i++) {
        r[i - a] = (int32_t)(by[i] / k);
        pos[by[i]] = base + (i - a);
      }
      for (int64_t i = b - a; i < chunk; i++) r[i] = r[0];
      j++;
    }
done:
  free(start);
  free(at);
  free(by);
  return rc;
}

/* The expert-contiguous dispatch the CUDA path builds (the first three steps of moe_plan, moe_host.cpp:203-215):
 * offsets[E + 1] (exclusive scan of the per-expert pair counts) and perm[i] = the i-th pair in expert-then-pair order,
 * slot[p] = the position of pair p in perm. */
int oracle_moe_dispatch(const int32_t* ids, int64_t n, int k, int E, int64_t* offsets, int32_t* perm, int32_t* slot) {
  const int64_t pairs = n * k;
  for (int x = 0; x <= E; x++) offsets[x] = 0;
  for (int64_t p = 0; p < pairs; p++) {
    if (ids[p] < 0 || ids[p] >= E) return ORACLE_EINVAL;
    offsets[ids[p] + 1]++;
  }
  for (int x = 0; x < E; x++) offsets[x + 1] += offsets[x];
  int64_t* at = (int64_t*)malloc(sizeof(int64_t) * ((size_t)E + 1));
  if (!at) return ORACLE_EINVAL;
  memcpy(at, offsets, sizeof(int64_t) * (size_t)E);
  for (int64_t p = 0; p < pairs; p++) {
    const int64_t i = at[ids[p]]++;
    perm[i] = (int32_t)p;
    slot[p] = (int32_t)i;
  }
  free(at);
  return ORACLE_OK;
}

/* ---- dequant (dequant.cpp:21-147), fp32 operations in the reference's order ---- */

static float f16(const uint8_t* p) { /* dequant.cpp:21-29 */
  uint16_t h;
  memcpy(&h, p, 2);
  const uint32_t s = (uint32_t)(h >> 15) << 31, e = (h >> 10) & 31, m = h & 1023;
  uint32_t u;
  float f;
  if (e == 31) {
    u = s | 0x7F800000u | m << 13;
    memcpy(&f, &u, 4);
    return f;
  }
  if (e) {
    u = s | (e + 112) << 23 | m << 13;
    memcpy(&f, &u, 4);
    return f;
  }
  const float v = (float)m * 0x1p-24f;
  return s ? -v : v;
}

static void q4_0(const uint8_t* b, float* o) { /* dequant.cpp:40-47: w = (q - 8) d */
  const float d = f16(b);
  for (int j = 0; j < 32; j++) {
    const int q = j < 16 ? b[2 + j] & 15 : b[2 + j - 16] >> 4;
    o[j] = ((float)q - 8.0f) * d;
  }
}

static void q4_1(const uint8_t* b, float* o) { /* dequant.cpp:49-56: w = d q + m */
  const float d = f16(b), m = f16(b + 2);
  for (int j = 0; j < 32; j++) {
    const int q = j < 16 ? b[4 + j] & 15 : b[4 + j - 16] >> 4;
    o[j] = d * (float)q + m;
  }
}

static void q8_0(const uint8_t* b, float* o) { /* dequant.cpp:58-62: w = d q */
  const float d = f16(b);
  for (int j = 0; j < 32; j++) o[j] = d * (float)(int8_t)b[2 + j];
}

/* Q4_K / Q5_K (dequant.cpp:64-81): 6-bit scales and mins of eight 32-groups packed in 12 bytes;
 * w = q (d sc_g) - dmin mn_g */
static void q45_k(const uint8_t* b, float* o, int q5) {
  const float d = f16(b), dmin = f16(b + 2);
  const uint8_t *lo = b + 4, *hi = b + 8, *top = b + 12, *qh = b + 16, *qs = b + (q5 ? 48 : 16);
  for (int g = 0; g < 8; g++) {
    const int sc = g < 4 ? lo[g] & 63 : (top[g - 4] & 15) | (lo[g - 4] >> 6) << 4;
    const int mn = g < 4 ? hi[g] & 63 : (top[g - 4] >> 4) | (hi[g - 4] >> 6) << 4;
    const float dsc = d * (float)sc, dmn = dmin * (float)mn;
    for (int l = 0; l < 32; l++) {
      const uint8_t c = qs[32 * (g >> 1) + l];
      const int q = (g & 1 ? c >> 4 : c & 15) | (q5 ? ((qh[l] >> g) & 1) << 4 : 0);
      const float t = (float)q * dsc;
      o[32 * g + l] = t - dmn;
    }
  }
}

static void q6_k(const uint8_t* b, float* o) { /* dequant.cpp:83-101: w = (q - 32) (sc_j d) */
  const uint8_t *ql = b, *qh = b + 128;
  const int8_t* sc = (const int8_t*)(b + 192);
  const float d = f16(b + 208);
  for (int h = 0; h < 2; h++)
    for (int jj = 0; jj < 4; jj++) {
      const uint8_t* c = ql + 64 * h + 32 * (jj & 1);
      const uint8_t* e = qh + 32 * h;
      const int sh = jj < 2 ? 0 : 4;
      float* out = o + 128 * h + 32 * jj;
      const float s0 = (float)sc[8 * h + 2 * jj] * d, s1 = (float)sc[8 * h + 2 * jj + 1] * d;
      for (int l = 0; l < 32; l++) {
        const int q = (((c[l] >> sh) & 15) | ((e[l] >> (2 * jj)) & 3) << 4) - 32;
        out[l] = (float)q * (l < 16 ? s0 : s1);
      }
    }
}

/* Q3_K (dequant.cpp:103-117): 110 B per 256 = hmask[32], qs[64], 12 scale bytes, d. Sixteen 16-value sub-blocks s,
 * each with a 6-bit scale (stored + 32): low nibble from byte s (s < 8) or the high nibble of byte s - 8, top two bits
 * from byte 8 + s % 4 at bit 2 (s / 4). Value v = 128 n + 32 j + i (i < 32): a 3-bit q = crumb j of qs[32 n + i] | bit
 * (4 n + j) of hmask[i] << 2; w = (d (scale - 32)) (q - 4). */
static void q3_k(const uint8_t* b, float* o) {
  const uint8_t *hm = b, *qs = b + 32, *sc = b + 96;
  const float d = f16(b + 108);
  for (int s = 0; s < 16; s++) {
    const int low = s < 8 ? sc[s] & 15 : sc[s - 8] >> 4, top = (sc[8 + (s & 3)] >> (2 * (s >> 2))) & 3;
    const float a = d * (float)((low | top << 4) - 32);
    const int n = s >> 3, j = (s >> 1) & 3;
    for (int l = 0; l < 16; l++) {
      const int i = 16 * (s & 1) + l;
      const int q = ((qs[32 * n + i] >> (2 * j)) & 3) | ((hm[i] >> (4 * n + j)) & 1) << 2;
      o[16 * s + l] = a * ((float)q - 4.0f);
    }
  }
}

/* the sixteen IQ4_NL / IQ4_XS code values (dequant.cpp:119, ggml's non-linear 4-bit grid) */
static const int8_t IQ4_GRID[16] = {-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113};

/* IQ4_NL (dequant.cpp:121-126): 18 B per 32, d then Q4_0's nibble layout; w = d grid[q] */
static void iq4_nl(const uint8_t* b, float* o) {
  const float d = f16(b);
  for (int l = 0; l < 16; l++) {
    o[l] = d * (float)IQ4_GRID[b[2 + l] & 15];
    o[16 + l] = d * (float)IQ4_GRID[b[2 + l] >> 4];
  }
}

/* IQ4_XS (dequant.cpp:128-140): 136 B per 256 = d, a u16 of high scale crumbs, 4 bytes of low scale nibbles, 8 x 16
 * code bytes. 32-group g: scale ls = nibble (g % 2) of byte 4 + g / 2 | crumb g of the u16 << 4; its codes in Q4_0's
 * layout at 8 + 16 g; w = (d (ls - 32)) grid[q] */
static void iq4_xs(const uint8_t* b, float* o) {
  const float d = f16(b);
  const int hi = b[2] | b[3] << 8;
  for (int g = 0; g < 8; g++) {
    const int ls = ((b[4 + (g >> 1)] >> (4 * (g & 1))) & 15) | ((hi >> (2 * g)) & 3) << 4;
    const float dl = d * (float)(ls - 32);
    const uint8_t* q = b + 8 + 16 * g;
    for (int l = 0; l < 16; l++) {
      o[32 * g + l] = dl * (float)IQ4_GRID[q[l] & 15];
      o[32 * g + 16 + l] = dl * (float)IQ4_GRID[q[l] >> 4];
    }
  }
}

static void f32_1(const uint8_t* b, float* o) { memcpy(o, b, 4); }
static void f16_1(const uint8_t* b, float* o) { *o = f16(b); }
static void bf16_1(const uint8_t* b, float* o) {
  uint16_t h;
  memcpy(&h, b, 2);
  const uint32_t u = (uint32_t)h << 16;
  memcpy(o, &u, 4);
}
static void q4_k(const uint8_t* b, float* o) { q45_k(b, o, 0); }
static void q5_k(const uint8_t* b, float* o) { q45_k(b, o, 1); }

typedef struct {
  const char* name;
  int per, bytes;
  void (*block)(const uint8_t*, float*);
} qtype_t;

/* dequant.cpp:154-157's table */
static const qtype_t TYPES[] = {{"F32", 1, 4, f32_1},      {"F16", 1, 2, f16_1},       {"BF16", 1, 2, bf16_1},
                                {"Q4_0", 32, 18, q4_0},    {"Q4_1", 32, 20, q4_1},     {"Q8_0", 32, 34, q8_0},
                                {"Q3_K", 256, 110, q3_k},  {"Q4_K", 256, 144, q4_k},   {"Q5_K", 256, 176, q5_k},
                                {"Q6_K", 256, 210, q6_k},  {"IQ4_NL", 32, 18, iq4_nl}, {"IQ4_XS", 256, 136, iq4_xs}};

int oracle_dequant_supported(const char* qtype) {
  for (size_t i = 0; i < sizeof(TYPES) / sizeof(TYPES[0]); i++)
    if (!strcmp(TYPES[i].name, qtype)) return 1;
  return 0;
}

/* dequant_rows (dequant.cpp:174-188): n rows row_bytes apart, their first cols values, into out (n x cols fp32) */
int oracle_dequant_rows(const char* qtype, const uint8_t* raw, int64_t n, int64_t row_bytes, int64_t cols,
                        float* out) {
  const qtype_t* t = NULL;
  for (size_t i = 0; i < sizeof(TYPES) / sizeof(TYPES[0]); i++)
    if (!strcmp(TYPES[i].name, qtype)) t = &TYPES[i];
  if (!t || cols % t->per || cols / t->per * t->bytes > row_bytes) return ORACLE_EINVAL;
  for (int64_t r = 0; r < n; r++)
    for (int64_t b = 0; b < cols / t->per; b++) t->block(raw + r * row_bytes + b * t->bytes, out + r * cols + b * t->per);
  return ORACLE_OK;
}
