/* rpg_oracle.c -- CPU restatement of the reference token loop (test oracle).
 * See rpg_oracle.h for what each part follows.  Build: oracle/Makefile
 * (gcc -O2 -ffp-contract=off).  Never linked into the engine.
 */
#define _GNU_SOURCE
#include "rpg_oracle.h"

#include <fcntl.h>
#include <float.h>
#include <math.h>
#include <pthread.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

/* ------------------------------------------------------------------ f16 */

float orc_f16_to_f32(uint16_t h) { /* src/dtypes.h:21-48 */
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t e = (h >> 10) & 0x1Fu, m = h & 0x3FFu, out;
  if (e == 0) {
    if (m == 0) {
      out = sign;
    } else {
      e = 127 - 15 + 1;
      while ((m & 0x400u) == 0) {
        m <<= 1;
        --e;
      }
      m &= 0x3FFu;
      out = sign | (e << 23) | (m << 13);
    }
  } else if (e == 31) {
    out = sign | 0x7F800000u | (m << 13);
  } else {
    out = sign | ((e + (127 - 15)) << 23) | (m << 13);
  }
  float f;
  memcpy(&f, &out, 4);
  return f;
}

uint16_t orc_f32_to_f16(float f) { /* round to nearest even */
  uint32_t x;
  memcpy(&x, &f, 4);
  uint32_t sign = (x >> 16) & 0x8000u, ax = x & 0x7FFFFFFFu;
  if (ax >= 0x7F800000u) return (uint16_t)(sign | 0x7C00u | (ax > 0x7F800000u ? 0x200u : 0u));
  if (ax >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u);
  if (ax < 0x38800000u) {
    if (ax < 0x33000000u) return (uint16_t)sign;
    uint32_t e = ax >> 23, mm = (ax & 0x7FFFFFu) | 0x800000u, shift = 126u - e;
    uint32_t q = mm >> shift, rem = mm & ((1u << shift) - 1u), half = 1u << (shift - 1u);
    if (rem > half || (rem == half && (q & 1u))) ++q;
    return (uint16_t)(sign | q);
  }
  uint32_t hh = (ax >> 13) - (112u << 10), rem = ax & 0x1FFFu;
  if (rem > 0x1000u || (rem == 0x1000u && (hh & 1u))) ++hh;
  return (uint16_t)(sign | hh);
}

static inline float half_at(const uint8_t* p) { return orc_f16_to_f32((uint16_t)(p[0] | (p[1] << 8))); }

/* ------------------------------------------------------------------ dequant */

static void get_scale_min_k4(int j, const uint8_t* q, uint8_t* d, uint8_t* m) { /* quant.cc:159-167 */
  if (j < 4) {
    *d = q[j] & 63;
    *m = q[j + 4] & 63;
  } else {
    *d = (uint8_t)((q[j + 4] & 0x0F) | ((q[j - 4] >> 6) << 4));
    *m = (uint8_t)((q[j + 4] >> 4) | ((q[j] >> 6) << 4));
  }
}

static void deq_q4k(const uint8_t* src, int64_t n, float* y) { /* quant.cc:252-277 */
  for (int64_t b = 0; b < n / 256; ++b) {
    const uint8_t* p = src + b * 144;
    const float d = half_at(p), dmin = half_at(p + 2);
    const uint8_t* sc = p + 4;
    const uint8_t* q = p + 16;
    int is = 0;
    for (int j = 0; j < 256; j += 64) {
      uint8_t s, m;
      get_scale_min_k4(is + 0, sc, &s, &m);
      const float d1 = d * (float)s, m1 = dmin * (float)m;
      get_scale_min_k4(is + 1, sc, &s, &m);
      const float d2 = d * (float)s, m2 = dmin * (float)m;
      for (int l = 0; l < 32; ++l) *y++ = d1 * (float)(q[l] & 0x0F) - m1;
      for (int l = 0; l < 32; ++l) *y++ = d2 * (float)(q[l] >> 4) - m2;
      q += 32;
      is += 2;
    }
  }
}

static void deq_q6k(const uint8_t* src, int64_t n, float* out) { /* quant.cc:321-354 */
  for (int64_t b = 0; b < n / 256; ++b) {
    const uint8_t* p = src + b * 210;
    const uint8_t* ql = p;
    const uint8_t* qh = p + 128;
    const int8_t* sc = (const int8_t*)(p + 192);
    const float d = half_at(p + 208);
    float* y = out + b * 256;
    for (int blk = 0; blk < 256; blk += 128) {
      for (int l = 0; l < 32; ++l) {
        const int is = l / 16;
        const int q1 = (int)((ql[l] & 0x0F) | (((qh[l] >> 0) & 3) << 4)) - 32;
        const int q2 = (int)((ql[l + 32] & 0x0F) | (((qh[l] >> 2) & 3) << 4)) - 32;
        const int q3 = (int)((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
        const int q4 = (int)((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
        y[l + 0] = d * (float)sc[is + 0] * (float)q1;
        y[l + 32] = d * (float)sc[is + 2] * (float)q2;
        y[l + 64] = d * (float)sc[is + 4] * (float)q3;
        y[l + 96] = d * (float)sc[is + 6] * (float)q4;
      }
      y += 128;
      ql += 64;
      qh += 32;
      sc += 8;
    }
  }
}

static void deq_q5k(const uint8_t* src, int64_t n, float* y) { /* quant.cc:281-313 */
  /* 176-byte block: d, dmin (fp16), 12 bytes of packed 6-bit scales/mins,
     32 bytes of fifth bits, 128 bytes of low nibbles; a 64-column group j
     takes nibble halves of qs[32 j ..) and bits 2j, 2j+1 of qh */
  for (int64_t b = 0; b < n / 256; ++b) {
    const uint8_t* p = src + b * 176;
    const float d = half_at(p), dmin = half_at(p + 2);
    const uint8_t* qh = p + 16;
    for (int j = 0; j < 4; ++j) {
      const uint8_t* ql = p + 48 + 32 * j;
      for (int half = 0; half < 2; ++half) {
        uint8_t s, m;
        get_scale_min_k4(2 * j + half, p + 4, &s, &m);
        const float dl = d * (float)s, ml = dmin * (float)m;
        const int bit = 2 * j + half;
        for (int l = 0; l < 32; ++l) {
          const int q = (half ? ql[l] >> 4 : ql[l] & 0x0F) + (((qh[l] >> bit) & 1) ? 16 : 0);
          *y++ = dl * (float)q - ml;
        }
      }
    }
  }
}

static void deq_q8_0(const uint8_t* src, int64_t n, float* y) { /* quant.cc:132-141 */
  /* 34-byte block of 32: fp16 scale, then 32 signed bytes */
  for (int64_t b = 0; b < n / 32; ++b) {
    const uint8_t* p = src + b * 34;
    const float d = half_at(p);
    for (int l = 0; l < 32; ++l) *y++ = (float)(int8_t)p[2 + l] * d;
  }
}

int orc_dequant_row(uint32_t type, const uint8_t* src, int64_t n, float* dst) {
  switch (type) {
    case 0: memcpy(dst, src, (size_t)n * 4); return 0;
    case 1:
      for (int64_t i = 0; i < n; ++i) dst[i] = half_at(src + 2 * i);
      return 0;
    case 8: if (n % 32) return -1; deq_q8_0(src, n, dst); return 0;
    case 12: if (n % 256) return -1; deq_q4k(src, n, dst); return 0;
    case 13: if (n % 256) return -1; deq_q5k(src, n, dst); return 0;
    case 14: if (n % 256) return -1; deq_q6k(src, n, dst); return 0;
    default: return -1;
  }
}

static int64_t row_bytes(uint32_t type, int64_t cols) {
  switch (type) {
    case 0: return cols * 4;
    case 1: return cols * 2;
    case 8: return cols / 32 * 34;
    case 12: return cols / 256 * 144;
    case 13: return cols / 256 * 176;
    case 14: return cols / 256 * 210;
    default: return -1;
  }
}

/* ------------------------------------------------------------------ threads */

typedef void (*range_fn)(void* ctx, int64_t a, int64_t b);
typedef struct {
  range_fn fn;
  void* ctx;
  int64_t a, b;
} job_t;

static void* job_main(void* p) {
  job_t* j = (job_t*)p;
  j->fn(j->ctx, j->a, j->b);
  return NULL;
}

static void parallel_for(int n_threads, int64_t n, range_fn fn, void* ctx) {
  if (n_threads <= 1 || n < 64) {
    fn(ctx, 0, n);
    return;
  }
  if (n_threads > 64) n_threads = 64;
  pthread_t th[64];
  job_t jobs[64];
  const int64_t per = (n + n_threads - 1) / n_threads;
  int started = 0;
  for (int i = 0; i < n_threads; ++i) {
    const int64_t a = i * per, b = a + per < n ? a + per : n;
    if (a >= b) break;
    jobs[i].fn = fn;
    jobs[i].ctx = ctx;
    jobs[i].a = a;
    jobs[i].b = b;
    if (pthread_create(&th[i], NULL, job_main, &jobs[i]) != 0) {
      fn(ctx, a, b);
      jobs[i].fn = NULL;
    }
    ++started;
  }
  for (int i = 0; i < started; ++i) {
    if (jobs[i].fn != NULL) pthread_join(th[i], NULL);
  }
}

/* ------------------------------------------------------------------ matvec */

typedef struct {
  uint32_t type;
  const uint8_t* w;
  int64_t cols, rb;
  const float* x;
  int64_t n_tok, ldx;
  float* out;
  int64_t ldo, out_off;
  int64_t rows;
} mv_ctx;

static void mv_range(void* p, int64_t a, int64_t b) {
  mv_ctx* c = (mv_ctx*)p;
  float* row = (float*)malloc((size_t)c->cols * sizeof(float));
  for (int64_t r = a; r < b; ++r) {
    orc_dequant_row(c->type, c->w + r * c->rb, c->cols, row);
    for (int64_t t = 0; t < c->n_tok; ++t) {
      const float* x = c->x + t * c->ldx;
      double acc = 0.0;
      for (int64_t k = 0; k < c->cols; ++k) acc += (double)row[k] * (double)x[k];
      c->out[t * c->ldo + c->out_off + r] = (float)acc;
    }
  }
  free(row);
}

/* Many tokens: the matrix is dequantised once into wf, then row blocks x
 * token blocks of double dot products (eight partial sums per product, so a
 * 2811-token prefill of the benchmark models takes minutes, not hours; the
 * order of the double additions is not part of any contract). */
typedef struct {
  const float* wf;
  int64_t cols;
  const float* x;
  int64_t n_tok, ldx;
  float* out;
  int64_t ldo, out_off;
  int64_t rows;
} mm_ctx;

enum { kMmRows = 32, kMmToks = 32 };

static void deq_range(void* p, int64_t a, int64_t b) {
  mv_ctx* c = (mv_ctx*)p;
  for (int64_t r = a; r < b; ++r) orc_dequant_row(c->type, c->w + r * c->rb, c->cols, (float*)c->out + r * c->cols);
}

static double dot8(const float* a, const float* b, int64_t n) {
  double s[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  int64_t k = 0;
  for (; k + 8 <= n; k += 8) {
    for (int j = 0; j < 8; ++j) s[j] += (double)a[k + j] * (double)b[k + j];
  }
  for (; k < n; ++k) s[0] += (double)a[k] * (double)b[k];
  return ((s[0] + s[1]) + (s[2] + s[3])) + ((s[4] + s[5]) + (s[6] + s[7]));
}

static void mm_range(void* p, int64_t a, int64_t b) {
  mm_ctx* c = (mm_ctx*)p;
  const int64_t tblocks = (c->n_tok + kMmToks - 1) / kMmToks;
  for (int64_t job = a; job < b; ++job) {
    const int64_t rb = job / tblocks, tb = job - rb * tblocks;
    const int64_t r0 = rb * kMmRows, r1 = r0 + kMmRows < c->rows ? r0 + kMmRows : c->rows;
    const int64_t t0 = tb * kMmToks, t1 = t0 + kMmToks < c->n_tok ? t0 + kMmToks : c->n_tok;
    for (int64_t t = t0; t < t1; ++t) {
      const float* x = c->x + t * c->ldx;
      for (int64_t r = r0; r < r1; ++r) c->out[t * c->ldo + c->out_off + r] = (float)dot8(c->wf + r * c->cols, x, c->cols);
    }
  }
}

static void matvec_into(uint32_t type, const uint8_t* w, int64_t rows, int64_t cols, const float* x,
                        int64_t n_tok, int64_t ldx, float* out, int64_t ldo, int64_t out_off, int n_threads) {
  mv_ctx c = {type, w, cols, row_bytes(type, cols), x, n_tok, ldx, out, ldo, out_off, rows};
  if (n_tok < 8) {
    parallel_for(n_threads, rows, mv_range, &c);
    return;
  }
  float* wf = (float*)malloc((size_t)rows * (size_t)cols * sizeof(float));
  if (wf == NULL) {
    parallel_for(n_threads, rows, mv_range, &c);
    return;
  }
  mv_ctx d = c;
  d.out = wf;
  parallel_for(n_threads, rows, deq_range, &d);
  mm_ctx m = {wf, cols, x, n_tok, ldx, out, ldo, out_off, rows};
  const int64_t jobs = ((rows + kMmRows - 1) / kMmRows) * ((n_tok + kMmToks - 1) / kMmToks);
  parallel_for(n_threads, jobs, mm_range, &m);
  free(wf);
}

int orc_matvec(uint32_t type, const uint8_t* w, int64_t rows, int64_t cols, const float* x, int64_t n_tok,
               float* out, int n_threads) {
  if (row_bytes(type, cols) < 0) return -1;
  matvec_into(type, w, rows, cols, x, n_tok, cols, out, rows, 0, n_threads);
  return 0;
}

/* ------------------------------------------------------------------ GGUF */

typedef struct {
  char name[96];
  uint32_t type;
  int64_t dims[4];
  int n_dims;
  const uint8_t* data;
} gtensor;

typedef struct {
  char key[96];
  double v;
} gmeta;

struct orc_model {
  int fd;
  uint8_t* base;
  int64_t size;
  gtensor* tensors;
  int n_tensors;
  gmeta* meta;
  int n_meta;
  int32_t n_layers, hidden, n_heads, n_kv, head_dim, ffn, vocab, context, rope_pos, eos;
  float rope_theta, eps;
  float* rope; /* [rope_pos][head_dim] */
};

typedef struct {
  const uint8_t* p;
  int64_t pos, n;
  int bad;
} rd;

static uint64_t rd_u(rd* r, int sz) {
  uint64_t v = 0;
  if (r->pos + sz > r->n) {
    r->bad = 1;
    return 0;
  }
  memcpy(&v, r->p + r->pos, (size_t)sz);
  r->pos += sz;
  return v;
}

static int scalar_size(uint32_t t) {
  switch (t) {
    case 0: case 1: case 7: return 1;
    case 2: case 3: return 2;
    case 4: case 5: case 6: return 4;
    case 10: case 11: case 12: return 8;
    default: return -1;
  }
}

static double scalar_value(rd* r, uint32_t t) {
  uint64_t u = rd_u(r, scalar_size(t));
  switch (t) {
    case 0: return (double)(uint8_t)u;
    case 1: return (double)(int8_t)u;
    case 2: return (double)(uint16_t)u;
    case 3: return (double)(int16_t)u;
    case 4: return (double)(uint32_t)u;
    case 5: return (double)(int32_t)u;
    case 6: { float f; uint32_t w = (uint32_t)u; memcpy(&f, &w, 4); return (double)f; }
    case 7: return (double)(u != 0);
    case 10: return (double)u;
    case 11: return (double)(int64_t)u;
    case 12: { double d; memcpy(&d, &u, 8); return d; }
    default: return 0.0;
  }
}

static double meta_get(const orc_model* m, const char* key, double def) {
  for (int i = 0; i < m->n_meta; ++i) {
    if (strcmp(m->meta[i].key, key) == 0) return m->meta[i].v;
  }
  return def;
}

static const gtensor* find_tensor(const orc_model* m, const char* name) {
  for (int i = 0; i < m->n_tensors; ++i) {
    if (strcmp(m->tensors[i].name, name) == 0) return &m->tensors[i];
  }
  return NULL;
}

void orc_model_close(orc_model* m) {
  if (!m) return;
  if (m->base) munmap(m->base, (size_t)m->size);
  if (m->fd >= 0) close(m->fd);
  free(m->tensors);
  free(m->meta);
  free(m->rope);
  free(m);
}

orc_model* orc_model_open(const char* path, int32_t max_pos, char* err, int errlen) {
#define FAIL(msg)                                    \
  do {                                               \
    if (err) snprintf(err, (size_t)errlen, "%s", msg); \
    orc_model_close(m);                              \
    return NULL;                                     \
  } while (0)
  orc_model* m = (orc_model*)calloc(1, sizeof(orc_model));
  m->fd = open(path, O_RDONLY);
  if (m->fd < 0) FAIL("cannot open the model file");
  struct stat st;
  fstat(m->fd, &st);
  m->size = st.st_size;
  m->base = (uint8_t*)mmap(NULL, (size_t)m->size, PROT_READ, MAP_PRIVATE, m->fd, 0);
  if (m->base == MAP_FAILED) {
    m->base = NULL;
    FAIL("mmap failed");
  }
  rd r = {m->base, 0, m->size, 0};
  if (rd_u(&r, 4) != 0x46554747u) FAIL("not a GGUF file");
  const uint32_t ver = (uint32_t)rd_u(&r, 4);
  const uint64_t nt = ver == 1 ? rd_u(&r, 4) : rd_u(&r, 8);
  const uint64_t nkv = ver == 1 ? rd_u(&r, 4) : rd_u(&r, 8);
  m->meta = (gmeta*)calloc(nkv + 1, sizeof(gmeta));
  char arch[32] = "";
  int64_t alignment = 32;
  for (uint64_t i = 0; i < nkv && !r.bad; ++i) {
    const uint64_t kl = rd_u(&r, 8);
    char key[96] = "";
    if (kl < sizeof(key)) memcpy(key, r.p + r.pos, kl);
    r.pos += (int64_t)kl;
    const uint32_t t = (uint32_t)rd_u(&r, 4);
    if (t == 8) {
      const uint64_t sl = rd_u(&r, 8);
      if (strcmp(key, "general.architecture") == 0 && sl < sizeof(arch)) memcpy(arch, r.p + r.pos, sl);
      r.pos += (int64_t)sl;
    } else if (t == 9) {
      const uint32_t et = (uint32_t)rd_u(&r, 4);
      const uint64_t cnt = rd_u(&r, 8);
      if (et == 8) {
        for (uint64_t k = 0; k < cnt && !r.bad; ++k) r.pos += (int64_t)rd_u(&r, 8);
      } else {
        r.pos += (int64_t)cnt * scalar_size(et);
      }
    } else {
      const double v = scalar_value(&r, t);
      snprintf(m->meta[m->n_meta].key, sizeof(m->meta[0].key), "%s", key);
      m->meta[m->n_meta++].v = v;
      if (strcmp(key, "general.alignment") == 0) alignment = (int64_t)v;
    }
  }
  if (r.bad) FAIL("truncated metadata");
  if (strcmp(arch, "qwen3") != 0) FAIL("architecture is not qwen3");
  m->tensors = (gtensor*)calloc(nt, sizeof(gtensor));
  uint64_t* offs = (uint64_t*)calloc(nt, sizeof(uint64_t));
  for (uint64_t i = 0; i < nt && !r.bad; ++i) {
    gtensor* t = &m->tensors[i];
    const uint64_t nl = rd_u(&r, 8);
    if (nl < sizeof(t->name)) memcpy(t->name, r.p + r.pos, nl);
    r.pos += (int64_t)nl;
    t->n_dims = (int)rd_u(&r, 4);
    for (int d = 0; d < t->n_dims && d < 4; ++d) t->dims[d] = (int64_t)rd_u(&r, 8);
    t->type = (uint32_t)rd_u(&r, 4);
    offs[i] = rd_u(&r, 8);
  }
  m->n_tensors = (int)nt;
  const int64_t start = (r.pos + alignment - 1) / alignment * alignment;
  for (uint64_t i = 0; i < nt; ++i) m->tensors[i].data = m->base + start + (int64_t)offs[i];
  free(offs);
  if (r.bad) FAIL("truncated tensor table");

  m->n_layers = (int32_t)meta_get(m, "qwen3.block_count", 0);
  m->hidden = (int32_t)meta_get(m, "qwen3.embedding_length", 0);
  m->n_heads = (int32_t)meta_get(m, "qwen3.attention.head_count", 0);
  m->n_kv = (int32_t)meta_get(m, "qwen3.attention.head_count_kv", m->n_heads);
  m->ffn = (int32_t)meta_get(m, "qwen3.feed_forward_length", 0);
  m->context = (int32_t)meta_get(m, "qwen3.context_length", 4096);
  m->head_dim = (int32_t)meta_get(m, "qwen3.attention.key_length", 0);
  if (m->head_dim <= 0 && m->n_heads > 0) m->head_dim = m->hidden / m->n_heads;
  m->rope_theta = (float)meta_get(m, "qwen3.rope.freq_base", 10000.0);
  m->eps = (float)meta_get(m, "qwen3.attention.layer_norm_rms_epsilon", 1e-6);
  m->eos = (int32_t)meta_get(m, "tokenizer.ggml.eos_token_id", -1);
  const gtensor* emb = find_tensor(m, "token_embd.weight");
  if (!emb) FAIL("token_embd.weight missing");
  m->vocab = (int32_t)emb->dims[1];
  if (m->n_layers <= 0 || m->hidden <= 0 || m->n_heads <= 0 || m->head_dim <= 0 || m->ffn <= 0)
    FAIL("incomplete metadata");

  /* RoPE table: src/gpu_model.cu:90-120 */
  m->rope_pos = max_pos < m->context ? max_pos : m->context;
  if (m->rope_pos <= 0) m->rope_pos = 1;
  const int half = m->head_dim / 2;
  m->rope = (float*)malloc((size_t)m->rope_pos * m->head_dim * sizeof(float));
  double* inv = (double*)malloc((size_t)half * sizeof(double));
  for (int i = 0; i < half; ++i) inv[i] = 1.0 / pow((double)m->rope_theta, (double)(2 * i) / (double)m->head_dim);
  for (int64_t p = 0; p < m->rope_pos; ++p) {
    float* row = m->rope + p * m->head_dim;
    for (int i = 0; i < half; ++i) {
      const double ang = (double)p * inv[i];
      row[i] = (float)cos(ang);
      row[half + i] = (float)sin(ang);
    }
  }
  free(inv);
  return m;
#undef FAIL
}

void orc_model_shape(const orc_model* m, int32_t* o) {
  o[0] = m->n_layers; o[1] = m->hidden; o[2] = m->n_heads; o[3] = m->n_kv; o[4] = m->head_dim;
  o[5] = m->ffn; o[6] = m->vocab; o[7] = m->context; o[8] = m->rope_pos; o[9] = m->eos;
}

/* ------------------------------------------------------------------ session */

struct orc_session {
  orc_model* m;
  int32_t max_seq;
  int n_threads;
  int64_t len;
  uint16_t* kc; /* [layer][kv][max_seq][hd] */
  uint16_t* vc;
  float* logits; /* last position */
  int logits_valid;
};

orc_session* orc_session_create(orc_model* m, int32_t max_seq, int n_threads) {
  if (max_seq <= 0 || max_seq > m->rope_pos) return NULL;
  orc_session* s = (orc_session*)calloc(1, sizeof(orc_session));
  s->m = m;
  s->max_seq = max_seq;
  s->n_threads = n_threads > 0 ? n_threads : (int)sysconf(_SC_NPROCESSORS_ONLN);
  const size_t n = (size_t)m->n_layers * m->n_kv * max_seq * m->head_dim;
  s->kc = (uint16_t*)calloc(n, 2);
  s->vc = (uint16_t*)calloc(n, 2);
  s->logits = (float*)calloc((size_t)m->vocab, sizeof(float));
  return s;
}

void orc_session_free(orc_session* s) {
  if (!s) return;
  free(s->kc);
  free(s->vc);
  free(s->logits);
  free(s);
}

int64_t orc_session_len(const orc_session* s) { return s->len; }
void orc_session_set_len(orc_session* s, int64_t len) {
  if (len != s->len) s->logits_valid = 0;
  s->len = len;
}

static const gtensor* layer_tensor(const orc_model* m, int l, const char* suffix) {
  char nm[96];
  snprintf(nm, sizeof(nm), "blk.%d.%s", l, suffix);
  return find_tensor(m, nm);
}

static void norm_vec(const float* w_raw, uint32_t wtype, int64_t n, float* w) { orc_dequant_row(wtype, (const uint8_t*)w_raw, n, w); }

/* RMSNorm: double sum of squares, scale = float(1/sqrt(mean + eps)), out = x*scale*w */
static void rmsnorm(const float* x, const float* w, int64_t n, float eps, float* out) {
  double ss = 0.0;
  for (int64_t i = 0; i < n; ++i) ss += (double)x[i] * (double)x[i];
  const float scale = (float)(1.0 / sqrt(ss / (double)n + (double)eps));
  for (int64_t i = 0; i < n; ++i) out[i] = x[i] * scale * w[i];
}

static void rope_apply(float* v, const float* row, int hd) {
  const int half = hd / 2;
  for (int i = 0; i < half; ++i) {
    const double a = v[i], b = v[i + half], c = row[i], s = row[half + i];
    v[i] = (float)(a * c - b * s);
    v[i + half] = (float)(b * c + a * s);
  }
}

typedef struct {
  orc_session* s;
  int layer;
  const float* q; /* [n][q_dim] normalised + rotated */
  float* out;     /* [n][q_dim] */
  int64_t pos0, n;
} attn_ctx;

/* f16 -> f32 of every bit pattern (the attention loops convert each cached
 * element; a table keeps long contexts fast) */
static float g_f16_table[65536];
static pthread_once_t g_f16_once = PTHREAD_ONCE_INIT;
static void f16_table_init(void) {
  for (uint32_t h = 0; h < 65536u; ++h) g_f16_table[h] = orc_f16_to_f32((uint16_t)h);
}

static void attn_range(void* p, int64_t a, int64_t b) {
  attn_ctx* c = (attn_ctx*)p;
  const orc_model* m = c->s->m;
  const int hd = m->head_dim, nh = m->n_heads, group = m->n_heads / m->n_kv;
  const double scale = (double)(1.0f / sqrtf((float)hd));
  double* sc = (double*)malloc((size_t)(c->pos0 + c->n) * sizeof(double));
  double* acc = (double*)malloc((size_t)hd * sizeof(double));
  const float* f16 = g_f16_table;
  for (int64_t job = a; job < b; ++job) {
    const int64_t t = job / nh;
    const int h = (int)(job % nh), kh = h / group;
    const int64_t pos = c->pos0 + t;
    const float* q = c->q + t * (int64_t)nh * hd + (int64_t)h * hd;
    const size_t lbase = ((size_t)c->layer * m->n_kv + kh) * c->s->max_seq * hd;
    double mx = -DBL_MAX;
    for (int64_t s = 0; s <= pos; ++s) {
      const uint16_t* k = c->s->kc + lbase + (size_t)s * hd;
      double dot = 0.0;
      for (int d = 0; d < hd; ++d) dot += (double)q[d] * (double)f16[k[d]];
      sc[s] = dot * scale;
      if (sc[s] > mx) mx = sc[s];
    }
    double sum = 0.0;
    for (int64_t s = 0; s <= pos; ++s) {
      sc[s] = exp(sc[s] - mx);
      sum += sc[s];
    }
    /* each acc[d] adds its terms in position order, as a per-dimension loop would */
    for (int d = 0; d < hd; ++d) acc[d] = 0.0;
    for (int64_t s = 0; s <= pos; ++s) {
      const uint16_t* v = c->s->vc + lbase + (size_t)s * hd;
      const double w = sc[s];
      for (int d = 0; d < hd; ++d) acc[d] += w * (double)f16[v[d]];
    }
    float* o = c->out + t * (int64_t)nh * hd + (int64_t)h * hd;
    for (int d = 0; d < hd; ++d) o[d] = (float)(acc[d] / sum);
  }
  free(acc);
  free(sc);
}

static float silu_mul(float g, float u) { return (float)(((double)g / (1.0 + exp(-(double)g))) * (double)u); }

int orc_prefill(orc_session* s, const int32_t* tokens, int64_t n, float* last_logits, float* hidden) {
  orc_model* m = s->m;
  if (n <= 0 || s->len + n > s->max_seq) return -1;
  for (int64_t t = 0; t < n; ++t) {
    if (tokens[t] < 0 || tokens[t] >= m->vocab) return -2;
  }
  const int64_t H = m->hidden, hd = m->head_dim, qd = (int64_t)m->n_heads * hd, kvd = (int64_t)m->n_kv * hd;
  const int64_t F = m->ffn, pos0 = s->len;
  float* x = (float*)malloc((size_t)(n * H) * 4);
  float* xn = (float*)malloc((size_t)(n * H) * 4);
  float* q = (float*)malloc((size_t)(n * qd) * 4);
  float* k = (float*)malloc((size_t)(n * kvd) * 4);
  float* v = (float*)malloc((size_t)(n * kvd) * 4);
  float* att = (float*)malloc((size_t)(n * qd) * 4);
  float* proj = (float*)malloc((size_t)(n * H) * 4);
  float* gate = (float*)malloc((size_t)(n * F) * 4);
  float* up = (float*)malloc((size_t)(n * F) * 4);
  float* nw = (float*)malloc((size_t)(H > F ? H : F) * 4);
  float* qn = (float*)malloc((size_t)hd * 4);
  float* kn = (float*)malloc((size_t)hd * 4);

  const gtensor* emb = find_tensor(m, "token_embd.weight");
  const int64_t erb = row_bytes(emb->type, H);
  for (int64_t t = 0; t < n; ++t) orc_dequant_row(emb->type, emb->data + (int64_t)tokens[t] * erb, H, x + t * H);
  if (hidden) memcpy(hidden, x, (size_t)(n * H) * 4);

  for (int l = 0; l < m->n_layers; ++l) {
    const gtensor* an = layer_tensor(m, l, "attn_norm.weight");
    const gtensor* fnw = layer_tensor(m, l, "ffn_norm.weight");
    const gtensor* qnw = layer_tensor(m, l, "attn_q_norm.weight");
    const gtensor* knw = layer_tensor(m, l, "attn_k_norm.weight");
    const gtensor* wq = layer_tensor(m, l, "attn_q.weight");
    const gtensor* wk = layer_tensor(m, l, "attn_k.weight");
    const gtensor* wv = layer_tensor(m, l, "attn_v.weight");
    const gtensor* wo = layer_tensor(m, l, "attn_output.weight");
    const gtensor* wg = layer_tensor(m, l, "ffn_gate.weight");
    const gtensor* wu = layer_tensor(m, l, "ffn_up.weight");
    const gtensor* wd = layer_tensor(m, l, "ffn_down.weight");
    norm_vec((const float*)an->data, an->type, H, nw);
    for (int64_t t = 0; t < n; ++t) rmsnorm(x + t * H, nw, H, m->eps, xn + t * H);
    matvec_into(wq->type, wq->data, qd, H, xn, n, H, q, qd, 0, s->n_threads);
    matvec_into(wk->type, wk->data, kvd, H, xn, n, H, k, kvd, 0, s->n_threads);
    matvec_into(wv->type, wv->data, kvd, H, xn, n, H, v, kvd, 0, s->n_threads);
    norm_vec((const float*)qnw->data, qnw->type, hd, qn);
    norm_vec((const float*)knw->data, knw->type, hd, kn);
    for (int64_t t = 0; t < n; ++t) {
      const float* rr = m->rope + (pos0 + t) * hd;
      for (int h = 0; h < m->n_heads; ++h) {
        float* qh = q + t * qd + (int64_t)h * hd;
        rmsnorm(qh, qn, hd, m->eps, qh);
        rope_apply(qh, rr, (int)hd);
      }
      for (int h = 0; h < m->n_kv; ++h) {
        float* kh = k + t * kvd + (int64_t)h * hd;
        rmsnorm(kh, kn, hd, m->eps, kh);
        rope_apply(kh, rr, (int)hd);
        const size_t base = (((size_t)l * m->n_kv + h) * s->max_seq + (size_t)(pos0 + t)) * hd;
        for (int d = 0; d < hd; ++d) {
          s->kc[base + d] = orc_f32_to_f16(kh[d]);
          s->vc[base + d] = orc_f32_to_f16(v[t * kvd + (int64_t)h * hd + d]);
        }
      }
    }
    pthread_once(&g_f16_once, f16_table_init);
    attn_ctx ac = {s, l, q, att, pos0, n};
    parallel_for(s->n_threads, n * m->n_heads, attn_range, &ac);
    matvec_into(wo->type, wo->data, H, qd, att, n, qd, proj, H, 0, s->n_threads);
    for (int64_t i = 0; i < n * H; ++i) x[i] += proj[i];
    norm_vec((const float*)fnw->data, fnw->type, H, nw);
    for (int64_t t = 0; t < n; ++t) rmsnorm(x + t * H, nw, H, m->eps, xn + t * H);
    matvec_into(wg->type, wg->data, F, H, xn, n, H, gate, F, 0, s->n_threads);
    matvec_into(wu->type, wu->data, F, H, xn, n, H, up, F, 0, s->n_threads);
    for (int64_t i = 0; i < n * F; ++i) gate[i] = silu_mul(gate[i], up[i]);
    matvec_into(wd->type, wd->data, H, F, gate, n, F, proj, H, 0, s->n_threads);
    for (int64_t i = 0; i < n * H; ++i) x[i] += proj[i];
    if (hidden) memcpy(hidden + (int64_t)(l + 1) * n * H, x, (size_t)(n * H) * 4);
  }
  const gtensor* on = find_tensor(m, "output_norm.weight");
  norm_vec((const float*)on->data, on->type, H, nw);
  rmsnorm(x + (n - 1) * H, nw, H, m->eps, xn);
  const gtensor* out = find_tensor(m, "output.weight");
  if (!out) out = emb;
  matvec_into(out->type, out->data, m->vocab, H, xn, 1, H, s->logits, m->vocab, 0, s->n_threads);
  if (last_logits) memcpy(last_logits, s->logits, (size_t)m->vocab * 4);
  s->len = pos0 + n;
  s->logits_valid = 1;
  free(x); free(xn); free(q); free(k); free(v); free(att); free(proj); free(gate); free(up); free(nw);
  free(qn); free(kn);
  return 0;
}

/* ------------------------------------------------------------------ sampler */

static uint64_t splitmix64(uint64_t x) { /* src/sampler_gpu.cu:42-47 */
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}

float orc_counter_uniform(uint64_t seed, uint64_t counter) { /* sampler_gpu.cu:49-56 */
  const uint32_t bits = (uint32_t)(splitmix64(seed + 0x9E3779B97F4A7C15ull * counter) >> 40);
  return (float)bits * (1.0f / 16777216.0f);
}

static uint32_t order_key(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
static float from_order_key(uint32_t k) {
  const uint32_t u = (k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

static int64_t argmax_first(const float* x, int64_t n) { /* ties -> lowest index */
  float bv = -INFINITY;
  int64_t bi = 0;
  for (int64_t i = 0; i < n; ++i) {
    if (x[i] > bv) {
      bv = x[i];
      bi = i;
    }
  }
  return bi;
}

void orc_filter_to_probs(const float* logits, int64_t n, float temperature, int32_t top_k, float top_p,
                         float* probs) { /* src/sampler_gpu.cu:161-290 */
  for (int64_t i = 0; i < n; ++i) probs[i] = logits[i];
  if (!(temperature > 0.0f)) {
    const int64_t best = argmax_first(probs, n);
    for (int64_t i = 0; i < n; ++i) probs[i] = 0.0f;
    probs[best] = 1.0f;
    return;
  }
  if (temperature != 1.0f) {
    const float inv = 1.0f / temperature;
    for (int64_t i = 0; i < n; ++i) probs[i] *= inv;
  }
  if (top_k > 1 && top_k < n) {
    uint32_t lo = 0u, hi = 0xFFFFFFFFu;
    while (lo < hi) {
      const uint32_t mid = (uint32_t)(lo + (((uint64_t)hi - lo + 1) >> 1));
      int64_t cnt = 0;
      for (int64_t i = 0; i < n; ++i) cnt += order_key(probs[i]) >= mid;
      if (cnt >= top_k) lo = mid; else hi = mid - 1;
    }
    const float kth = from_order_key(lo);
    for (int64_t i = 0; i < n; ++i) {
      if (probs[i] < kth) probs[i] = -INFINITY;
    }
  }
  float mx = -INFINITY;
  for (int64_t i = 0; i < n; ++i) mx = probs[i] > mx ? probs[i] : mx;
  double sum = 0.0;
  for (int64_t i = 0; i < n; ++i) {
    const float e = expf(probs[i] - mx);
    probs[i] = e;
    sum += (double)e;
  }
  const float inv = (float)(1.0 / sum);
  for (int64_t i = 0; i < n; ++i) probs[i] *= inv;
  if (top_p > 0.0f && top_p < 1.0f) {
    const double threshold = 1.0 - (double)top_p;
    uint32_t lo = 0u, hi = 0xFFFFFFFFu;
    while (lo < hi) {
      const uint32_t mid = (uint32_t)(lo + (((uint64_t)hi - lo + 1) >> 1));
      double s = 0.0;
      for (int64_t i = 0; i < n; ++i) {
        if (order_key(probs[i]) <= mid) s += (double)probs[i];
      }
      if (s <= threshold) lo = mid; else hi = mid - 1;
    }
    const float cut = from_order_key(lo);
    for (int64_t i = 0; i < n; ++i) {
      if (probs[i] <= cut) probs[i] = 0.0f;
    }
    const int64_t best = argmax_first(probs, n);
    if (probs[best] == 0.0f) probs[best] = 1.0f;
    double s2 = 0.0;
    for (int64_t i = 0; i < n; ++i) s2 += (double)probs[i];
    if (s2 > 0.0) {
      const float inv2 = (float)(1.0 / s2);
      for (int64_t i = 0; i < n; ++i) probs[i] *= inv2;
    }
  }
}

int32_t orc_sample_token(const float* logits, int64_t n, float temperature, int32_t top_k, float top_p,
                         float u) { /* sampler_gpu.cu:312-336, 427-440 */
  if (!(temperature > 0.0f)) return (int32_t)argmax_first(logits, n);
  float* probs = (float*)malloc((size_t)n * sizeof(float));
  orc_filter_to_probs(logits, n, temperature, top_k, top_p, probs);
  double cum = 0.0;
  int32_t tok = -1;
  for (int64_t i = 0; i < n; ++i) {
    cum += (double)probs[i];
    if (cum > (double)u) {
      tok = (int32_t)i;
      break;
    }
  }
  if (tok < 0) {
    float bv = probs[0];
    tok = 0;
    for (int64_t i = 1; i < n; ++i) {
      if (probs[i] > bv) {
        bv = probs[i];
        tok = (int32_t)i;
      }
    }
  }
  free(probs);
  return tok;
}

/* ------------------------------------------------------------------ generate */

int orc_generate(orc_session* s, float temperature, int32_t top_k, float top_p, uint64_t seed, int32_t max_tokens,
                 const int32_t* stop, int32_t n_stop, int32_t* out, float* step_logits) {
  const int32_t V = s->m->vocab;
  if (!s->logits_valid || max_tokens <= 0) return -1;
  int produced = 0;
  for (int i = 0; i < max_tokens; ++i) {
    if (s->len >= s->max_seq) return -2;
    const uint64_t counter = (uint64_t)s->len;
    const float u = orc_counter_uniform(seed, counter);
    const int32_t next = orc_sample_token(s->logits, V, temperature, top_k, top_p, u);
    if (step_logits) memcpy(step_logits + (int64_t)i * V, s->logits, (size_t)V * 4);
    out[produced++] = next;
    int is_stop = 0;
    for (int j = 0; j < n_stop; ++j) is_stop |= stop[j] == next;
    if (orc_prefill(s, &next, 1, NULL, NULL) != 0) return -3;
    if (is_stop) break;
  }
  return produced;
}
