/*
 * CPU oracle of the packed-embedding codec.  TEST INFRASTRUCTURE ONLY: the
 * checker the CUDA codec is compared against (tests/ and bench.py's CPU legs);
 * nothing in the product path links or calls it.
 *
 * It restates, in plain C with f32 arithmetic in the reference's order (built
 * with -ffp-contract=off, so no product is fused into a sum):
 *   - embeddings_to_packed   src/packops.rs:172-301
 *   - embeddings_from_packed src/packops.rs:303-438
 *   - scale_histogram        src/packops.rs:31-103
 *   - Haar with mirrored odd edges, forward / inverse   src/haarops.rs:1-70
 *   - rANS64 (single stream, 32-bit renormalisation, bitstream of ryg_rans'
 *     public-domain rans64.h, as ported at src/rans64.rs:1-309)
 *
 * Stream layout (native = little-endian): u32 rows; per window of at most
 * 1024 rows: cols bytes of inverse column permutation, u16 symbol count,
 * (u16 symbol, u16 frequency) pairs in symbol order, u16 rANS byte count
 * (the reference's `as u16`, so it wraps above 65535), the rANS bytes.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define MAX_WINDOW_ROWS 1024
#define RANS_BITS 12
#define RANS64_L (1ull << 31)
static const float kRange = 29.0f;
static const float kInvSqrt2 = 0.7071067811865475f;

/* src/haarops.rs:4-30 */
static void haar_forward(float* x, int n0, float* tmp) {
  int n = n0;
  while (n > 1) {
    const int pairs = n / 2, odd = n & 1, nc = pairs + odd;
    for (int i = 0; i < pairs; ++i) {
      const float a = x[2 * i], b = x[2 * i + 1];
      tmp[i] = (a + b) * kInvSqrt2;
      tmp[nc + i] = (a - b) * kInvSqrt2;
    }
    if (odd) {
      const float a = x[n - 1];
      tmp[pairs] = (a + a) * kInvSqrt2;
    }
    memcpy(x, tmp, (size_t)n * sizeof(float));
    n = nc;
  }
}

/* src/haarops.rs:32-70 */
static void haar_inverse(float* x, int n0, float* tmp) {
  int levels[40];
  int nl = 0, n = n0;
  levels[nl++] = n;
  while (n > 1) {
    n = n / 2 + (n & 1);
    levels[nl++] = n;
  }
  for (int w = nl - 1; w >= 1; --w) {
    const int n_prev = levels[w - 1];
    const int odd = n_prev & 1, pairs = n_prev / 2, nc = pairs + odd;
    for (int i = 0; i < pairs; ++i) {
      const float s = x[i], d = x[nc + i];
      tmp[2 * i] = (s + d) * kInvSqrt2;
      tmp[2 * i + 1] = (s - d) * kInvSqrt2;
    }
    if (odd) tmp[n_prev - 1] = x[nc - 1] * kInvSqrt2;
    memcpy(x, tmp, (size_t)n_prev * sizeof(float));
  }
}

/* src/packops.rs:31-103.  sym/cnt: m (symbol, count) pairs in symbol order;
 * writes freq[m] summing to 1 << log2_scale.  Returns 0, or -1 when m does
 * not fit (the reference asserts). */
static int scale_histogram(const uint32_t* cnt, int m, int log2_scale, uint32_t* freq, uint64_t* rem, int* order) {
  const uint32_t target = 1u << log2_scale;
  if (m <= 0 || (uint32_t)m > target) return -1;
  const uint32_t remaining = target - (uint32_t)m;
  uint64_t sum = 0;
  for (int i = 0; i < m; ++i) sum += cnt[i];
  uint32_t acc = 0;
  for (int i = 0; i < m; ++i) {
    const uint64_t num = (uint64_t)cnt[i] * remaining;
    const uint32_t q = (uint32_t)(num / sum);
    rem[i] = num % sum;
    freq[i] = 1 + q;
    acc += q;
  }
  const uint32_t deficit = remaining - acc;
  if (deficit > 0) {
    /* stable sort of the indices by remainder, largest first */
    for (int i = 0; i < m; ++i) order[i] = i;
    for (int i = 1; i < m; ++i) {
      const int v = order[i];
      int j = i - 1;
      while (j >= 0 && rem[order[j]] < rem[v]) {
        order[j + 1] = order[j];
        --j;
      }
      order[j + 1] = v;
    }
    for (uint32_t k = 0; k < deficit && k < (uint32_t)m; ++k) freq[order[k]] += 1;
  }
  int64_t total = 0;
  for (int i = 0; i < m; ++i) total += freq[i];
  if (total != (int64_t)target) {
    int max_idx = 0; /* Iterator::max_by_key keeps the last of equal maxima */
    for (int i = 1; i < m; ++i)
      if (freq[i] >= freq[max_idx]) max_idx = i;
    while (total < (int64_t)target) {
      freq[max_idx] += 1;
      ++total;
    }
    while (total > (int64_t)target && freq[max_idx] > 1) {
      freq[max_idx] -= 1;
      --total;
    }
  }
  return 0;
}

/* rANS64 encoder symbol, src/rans64.rs:28-82 */
typedef struct {
  uint64_t x_max, rcp_freq, bias;
  uint32_t cmpl_freq, rcp_shift;
} EncSym;

static EncSym enc_symbol(uint32_t cum, uint32_t freq, uint32_t bits) {
  EncSym s;
  s.x_max = ((RANS64_L >> bits) << 32) * (uint64_t)freq;
  s.cmpl_freq = (1u << bits) - freq;
  if (freq < 2) {
    s.rcp_freq = ~0ull;
    s.rcp_shift = 0;
    s.bias = (uint64_t)cum + ((1ull << bits) - 1);
  } else {
    uint32_t shift = 0;
    while (freq > (1u << shift)) ++shift;
    const unsigned __int128 num = (unsigned __int128)1 << (shift + 63);
    s.rcp_freq = (uint64_t)((num + freq - 1) / freq);
    s.rcp_shift = shift - 1;
    s.bias = cum;
  }
  return s;
}

/* Encodes n symbols in order into buf[0, cap) from the back (src/rans64.rs:
 * 88-166); returns the start index of the stream, or -1 on overflow. */
static int64_t rans_encode(const uint16_t* qs, int64_t n, const EncSym* q2sym, uint8_t* buf, int64_t cap) {
  uint64_t x = RANS64_L;
  int64_t idx = cap;
  for (int64_t k = 0; k < n; ++k) {
    const EncSym* s = &q2sym[qs[k]];
    while (x >= s->x_max) {
      if (idx < 4) return -1;
      idx -= 4;
      const uint32_t v = (uint32_t)x;
      buf[idx] = (uint8_t)v;
      buf[idx + 1] = (uint8_t)(v >> 8);
      buf[idx + 2] = (uint8_t)(v >> 16);
      buf[idx + 3] = (uint8_t)(v >> 24);
      x >>= 32;
    }
    const uint64_t q = (uint64_t)(((unsigned __int128)x * s->rcp_freq) >> 64) >> s->rcp_shift;
    x = x + s->bias + q * s->cmpl_freq;
  }
  if (idx < 8) return -1;
  idx -= 8;
  for (int i = 0; i < 8; ++i) buf[idx + i] = (uint8_t)(x >> (8 * i));
  return idx;
}

static void put16(uint8_t* p, uint16_t v) {
  p[0] = (uint8_t)v;
  p[1] = (uint8_t)(v >> 8);
}
static uint16_t get16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }

/* Symbol of one scaled coefficient (src/packops.rs:245-250). */
static uint16_t coef_symbol(float x) {
  const float q = roundf(kRange * x);
  const float sf = 2.0f * fabsf(q) + (q < 0.0f ? 1.0f : 0.0f);
  const uint64_t s = sf >= 18446744073709551615.0f ? UINT64_MAX : (uint64_t)sf; /* `as usize` saturates */
  return (uint16_t)(s > 0 ? s - 1 : 0);
}

/* Upper bound of the packed size of `rows` x `cols` embeddings. */
int64_t oracle_packed_bound(int64_t rows, int cols) {
  int64_t b = 4;
  for (int64_t r = 0; r < rows; r += MAX_WINDOW_ROWS) {
    const int64_t w = rows - r < MAX_WINDOW_ROWS ? rows - r : MAX_WINDOW_ROWS;
    b += cols + 2 + 4 * 4096 + 2 + 2 * w * cols;
  }
  return b;
}

/* embeddings_to_packed: emb [rows][cols] f32 -> out; returns the byte count,
 * or -1 (cols > 255, rows == 0 or > 2^32 - 1, more than 4096 distinct symbols
 * in a window, encoder overflow or out too small). */
int64_t oracle_pack(const float* emb, int64_t rows, int cols, uint8_t* out, int64_t cap) {
  if (cols <= 0 || cols > 255 || rows <= 0 || rows > 0xFFFFFFFFll || cap < 4) return -1;
  const int64_t wmax = rows < MAX_WINDOW_ROWS ? rows : MAX_WINDOW_ROWS;
  float* raw = malloc(sizeof(float) * wmax * cols);
  float* tmp = malloc(sizeof(float) * (wmax > cols ? wmax : cols));
  float* colbuf = malloc(sizeof(float) * wmax);
  uint16_t* qs = malloc(sizeof(uint16_t) * wmax * cols);
  uint8_t* enc = malloc((size_t)(2 * wmax * cols));
  uint32_t* hist = malloc(sizeof(uint32_t) * 65536);
  uint32_t cnt[4097], freq[4097];
  uint16_t syms[4097];
  uint64_t rem[4097];
  int order[4097];
  EncSym* q2sym = malloc(sizeof(EncSym) * 65536);
  int64_t pos = 0, ret = -1;
  out[0] = (uint8_t)rows;
  out[1] = (uint8_t)(rows >> 8);
  out[2] = (uint8_t)(rows >> 16);
  out[3] = (uint8_t)(rows >> 24);
  pos = 4;
  for (int64_t off = 0; off < rows; off += MAX_WINDOW_ROWS) {
    const int64_t wr = rows - off < MAX_WINDOW_ROWS ? rows - off : MAX_WINDOW_ROWS;
    memcpy(raw, emb + off * cols, sizeof(float) * wr * cols);
    /* column sums and the ascending stable column order */
    float sums[256];
    int perm[256], inv[256];
    for (int c = 0; c < cols; ++c) sums[c] = 0.0f;
    for (int64_t r = 0; r < wr; ++r)
      for (int c = 0; c < cols; ++c) sums[c] += raw[r * cols + c];
    for (int c = 0; c < cols; ++c) perm[c] = c;
    for (int i = 1; i < cols; ++i) {
      const int v = perm[i];
      int j = i - 1;
      while (j >= 0 && sums[perm[j]] > sums[v]) {
        perm[j + 1] = perm[j];
        --j;
      }
      perm[j + 1] = v;
    }
    for (int c = 0; c < cols; ++c) inv[perm[c]] = c;
    if (pos + cols > cap) goto done;
    for (int c = 0; c < cols; ++c) out[pos++] = (uint8_t)inv[c];
    float rowbuf[256];
    for (int64_t r = 0; r < wr; ++r) {
      for (int c = 0; c < cols; ++c) rowbuf[c] = raw[r * cols + perm[c]];
      memcpy(raw + r * cols, rowbuf, sizeof(float) * cols);
    }
    for (int64_t r = 0; r < wr; ++r) haar_forward(raw + r * cols, cols, tmp);
    for (int c = 0; c < cols; ++c) {
      for (int64_t r = 0; r < wr; ++r) colbuf[r] = raw[r * cols + c];
      haar_forward(colbuf, (int)wr, tmp);
      for (int64_t r = 0; r < wr; ++r) raw[r * cols + c] = colbuf[r];
    }
    float abs_max = 0.00001f;
    for (int64_t i = 0; i < wr * cols; ++i) {
      const float a = fabsf(raw[i]);
      if (a < 1.0f && a > abs_max) abs_max = a;
    }
    const float inv_max = 1.0f / abs_max;
    uint16_t max_symbol = 0;
    for (int64_t i = 0; i < wr * cols; ++i) {
      const uint16_t s = coef_symbol(raw[i] * inv_max);
      qs[i] = s;
      if (s > max_symbol) max_symbol = s;
    }
    memset(hist, 0, sizeof(uint32_t) * ((size_t)max_symbol + 1));
    for (int64_t i = 0; i < wr * cols; ++i) hist[qs[i]]++;
    int m = 0;
    for (int s = 0; s <= max_symbol; ++s) {
      if (hist[s] > 0) {
        if (m == 4096) goto done;
        syms[m] = (uint16_t)s;
        cnt[m] = hist[s];
        ++m;
      }
    }
    if (scale_histogram(cnt, m, RANS_BITS, freq, rem, order) != 0) goto done;
    if (pos + 2 + 4 * m > cap) goto done;
    put16(out + pos, (uint16_t)m);
    pos += 2;
    uint32_t cum = 0;
    for (int i = 0; i < m; ++i) {
      q2sym[syms[i]] = enc_symbol(cum, freq[i], RANS_BITS);
      put16(out + pos, syms[i]);
      put16(out + pos + 2, (uint16_t)freq[i]);
      pos += 4;
      cum += freq[i];
    }
    const int64_t ecap = 2 * wr * cols;
    const int64_t start = rans_encode(qs, wr * cols, q2sym, enc, ecap);
    if (start < 0) goto done;
    const int64_t len = ecap - start;
    if (pos + 2 + len > cap) goto done;
    put16(out + pos, (uint16_t)len);
    pos += 2;
    memcpy(out + pos, enc + start, (size_t)len);
    pos += len;
  }
  ret = pos;
done:
  free(raw);
  free(tmp);
  free(colbuf);
  free(qs);
  free(enc);
  free(hist);
  free(q2sym);
  return ret;
}

/* embeddings_from_packed: returns the row count (out holds rows x cols f32,
 * L2-normalised), or -1 on a malformed stream (the reference's errors);
 * out_cap is in floats. */
int64_t oracle_unpack(const uint8_t* buf, int64_t len, int cols, float* out, int64_t out_cap) {
  if (len < 4 || cols <= 0 || cols > 255) return -1;
  const int64_t rows = (int64_t)buf[0] | ((int64_t)buf[1] << 8) | ((int64_t)buf[2] << 16) | ((int64_t)buf[3] << 24);
  if (rows * cols > out_cap) return -1;
  const float scale = 1.0f / kRange;
  int64_t pos = 4;
  float* tmp = malloc(sizeof(float) * (MAX_WINDOW_ROWS > cols ? MAX_WINDOW_ROWS : cols));
  float* colbuf = malloc(sizeof(float) * MAX_WINDOW_ROWS);
  float* cum2float = malloc(sizeof(float) * (1 << RANS_BITS));
  uint32_t* cum_start = malloc(sizeof(uint32_t) * (1 << RANS_BITS));
  uint32_t* cum_freq = malloc(sizeof(uint32_t) * (1 << RANS_BITS));
  int64_t ret = -1;
  for (int64_t off = 0; off < rows; off += MAX_WINDOW_ROWS) {
    const int64_t wr = rows - off < MAX_WINDOW_ROWS ? rows - off : MAX_WINDOW_ROWS;
    if (pos + cols + 2 > len) goto done;
    const uint8_t* idxs = buf + pos;
    pos += cols;
    for (int c = 0; c < cols; ++c)
      if (idxs[c] >= cols) goto done;
    const int n_sym = get16(buf + pos);
    pos += 2;
    if (pos + 4 * n_sym > len) goto done;
    const uint8_t* pairs = buf + pos;
    pos += 4 * n_sym;
    for (int c = 0; c < (1 << RANS_BITS); ++c) {
      cum2float[c] = 0.0f;
      cum_start[c] = 0;
      cum_freq[c] = 1;
    }
    uint32_t cum = 0;
    for (int i = 0; i < n_sym; ++i) {
      const uint16_t q = get16(pairs + 4 * i);
      const uint32_t f = get16(pairs + 4 * i + 2);
      if (cum > (1u << 31) || f > (1u << 31) - cum) goto done;
      float v = 0.0f;
      if (q != 0) {
        const uint16_t q1 = (uint16_t)(q + 1);
        const float sign = (q1 & 1) ? -1.0f : 1.0f;
        v = scale * sign * (float)(q1 >> 1);
      }
      for (uint32_t c = cum; c < cum + f; ++c) {
        if (c >= (1u << RANS_BITS)) goto done; /* the reference would index out of range */
        cum2float[c] = v;
        cum_start[c] = cum;
        cum_freq[c] = f;
      }
      cum += f;
    }
    if (pos + 2 > len) goto done;
    const int64_t csize = get16(buf + pos);
    pos += 2;
    if (pos + csize > len || csize < 8) goto done;
    const uint8_t* d = buf + pos;
    pos += csize;
    uint64_t x = 0;
    for (int i = 0; i < 8; ++i) x |= (uint64_t)d[i] << (8 * i);
    int64_t di = 8;
    float* t = out + off * cols;
    const uint64_t mask = (1ull << RANS_BITS) - 1;
    for (int64_t i = wr * cols - 1; i >= 0; --i) {
      const uint32_t c = (uint32_t)(x & mask);
      t[i] = cum2float[c];
      x = (uint64_t)cum_freq[c] * (x >> RANS_BITS) + (x & mask) - cum_start[c];
      if (x < RANS64_L) {
        if (di + 4 > csize) goto done;
        const uint64_t v = (uint64_t)d[di] | ((uint64_t)d[di + 1] << 8) | ((uint64_t)d[di + 2] << 16) |
                           ((uint64_t)d[di + 3] << 24);
        di += 4;
        x = (x << 32) | v;
        if (x < RANS64_L) goto done;
      }
    }
    for (int64_t r = 0; r < wr; ++r) haar_inverse(t + r * cols, cols, tmp);
    for (int c = 0; c < cols; ++c) {
      for (int64_t r = 0; r < wr; ++r) colbuf[r] = t[r * cols + c];
      haar_inverse(colbuf, (int)wr, tmp);
      for (int64_t r = 0; r < wr; ++r) t[r * cols + c] = colbuf[r];
    }
    float rowbuf[256];
    for (int64_t r = 0; r < wr; ++r) {
      for (int c = 0; c < cols; ++c) rowbuf[c] = t[r * cols + idxs[c]];
      memcpy(t + r * cols, rowbuf, sizeof(float) * cols);
    }
  }
  if (pos != len) goto done;
  for (int64_t r = 0; r < rows; ++r) {
    float* row = out + r * cols;
    float ss = 0.0f;
    for (int c = 0; c < cols; ++c) ss += row[c] * row[c];
    const float inv = 1.0f / sqrtf(ss);
    for (int c = 0; c < cols; ++c) row[c] *= inv;
  }
  ret = rows;
done:
  free(tmp);
  free(colbuf);
  free(cum2float);
  free(cum_start);
  free(cum_freq);
  return ret;
}
