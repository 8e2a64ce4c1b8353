/*
 * bm_oracle.c — TEST INFRASTRUCTURE. The CPU oracle for the layer-op kernels.
 *
 * A plain-C restatement of the double-precision check loops that the reference
 * (NolanKisser/BareMetalInferenceEngine) uses to verify its kernels, extended to
 * many rows, GQA heads, sequences and bf16 storage. Only the tests, the smoke
 * check and the benchmark's CPU-baseline leg use it, always as the checker or
 * as the timed CPU baseline; the product path never calls it.
 *
 * Storage dtype: 0 = fp32, 1 = bf16 (uint16 bit patterns). Inputs are widened
 * to double exactly; every result is computed in double and rounded once to the
 * storage type (bf16: round-to-nearest-even, through round-to-odd fp32).
 *
 * Functions and the reference code each one restates:
 *   oracle_rmsnorm      tests/kernel_tests.cu:75-79 (test_rms_norm), per row
 *   oracle_add          tests/kernel_tests.cu:206 (test_add): a[i] + b[i] in fp32
 *   oracle_add_rmsnorm  the add loop, then the RMSNorm loop on the stored sum
 *                       (src/execution_engine.cu:118,121)
 *   oracle_swiglu       tests/kernel_tests.cu:122 (test_swiglu)
 *   oracle_rope         tests/kernel_tests.cu:175-187 (reference_rope), per row
 *   oracle_kv_store     tests/kernel_tests.cu:223-226 (test_kv_store), per row
 *                       with a sequence dimension
 *   oracle_rope_kv_store  reference_rope on q and k, then the kv_store loop for
 *                       k and v (src/execution_engine.cu:113-115)
 *   oracle_gather       the row copy of src/execution_engine.cu:98-99 with the
 *                       id check of src/execution_engine.cu:63-65
 *   oracle_decode_attention  tests/kernel_tests.cu:229-258 (test_attention), batched, GQA
 *   oracle_gemm         tests/kernel_tests.cu:49-59 (reference_gemm)
 *   oracle_softmax      tests/kernel_tests.cu:105-160 (the softmax checks): per vector,
 *                       exp(x - max) / sum exp(x - max) in double
 *   oracle_gemm_swiglu  reference_gemm twice, then the SwiGLU of :122
 *                       (src/execution_engine.cu:122-124)
 *   oracle_layer_step(_mt)  the five ops above (or a chosen subset) over a row
 *                       range, single- or multi-threaded: the timed CPU baseline.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define BAD_ID 0x1
#define BAD_POSITION 0x2
#define BAD_SEQUENCE 0x4

/* ------------------------------------------------------------------------- */
/* bf16 helpers                                                               */

static inline float bits_to_f32(uint32_t b) {
  float f;
  memcpy(&f, &b, 4);
  return f;
}
static inline uint32_t f32_to_bits(float f) {
  uint32_t b;
  memcpy(&b, &f, 4);
  return b;
}

uint16_t oracle_f32_to_bf16(float f) {
  uint32_t b = f32_to_bits(f);
  if ((b & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((b >> 16) | 0x40u); /* quiet NaN */
  b += 0x7fffu + ((b >> 16) & 1u);
  return (uint16_t)(b >> 16);
}

float oracle_bf16_to_f32(uint16_t h) { return bits_to_f32((uint32_t)h << 16); }

/* double -> fp32 rounded to odd: keeps enough information for a second,
 * correct rounding to any narrower type. */
static float f64_to_f32_odd(double x) {
  float f = (float)x;
  if (isnan(x) || isinf(f) || (double)f == x) return f;
  if (fabs((double)f) > fabs(x)) f = nextafterf(f, 0.0f); /* truncate toward zero */
  uint32_t b = f32_to_bits(f) | 1u;
  return bits_to_f32(b);
}

uint16_t oracle_f64_to_bf16(double x) { return oracle_f32_to_bf16(f64_to_f32_odd(x)); }

static inline double ld(const void* p, int64_t i, int dt) {
  return dt == 0 ? (double)((const float*)p)[i] : (double)oracle_bf16_to_f32(((const uint16_t*)p)[i]);
}
static inline float ldf(const void* p, int64_t i, int dt) {
  return dt == 0 ? ((const float*)p)[i] : oracle_bf16_to_f32(((const uint16_t*)p)[i]);
}
static inline void st(void* p, int64_t i, double x, int dt) {
  if (dt == 0) {
    ((float*)p)[i] = (float)x;
  } else {
    ((uint16_t*)p)[i] = oracle_f64_to_bf16(x);
  }
}
static inline void stf(void* p, int64_t i, float x, int dt) {
  if (dt == 0) {
    ((float*)p)[i] = x;
  } else {
    ((uint16_t*)p)[i] = oracle_f32_to_bf16(x);
  }
}
static inline size_t esize(int dt) { return dt == 0 ? 4 : 2; }

/* ------------------------------------------------------------------------- */
/* RMSNorm (tests/kernel_tests.cu:75-79):                                     */
/*   sum_of_squares += (double)v * v; scale = 1 / sqrt(ss / size + eps);      */
/*   want[i] = (float)(in[i] * scale * weight[i])                              */

static void rmsnorm_row(void* out, const void* in, const void* w, int64_t dim, double eps, int dt) {
  double ss = 0.0;
  for (int64_t i = 0; i < dim; ++i) {
    const double v = ld(in, i, dt);
    ss += v * v;
  }
  const double scale = 1.0 / sqrt(ss / (double)dim + eps);
  for (int64_t i = 0; i < dim; ++i) st(out, i, ld(in, i, dt) * scale * ld(w, i, dt), dt);
}

void oracle_rmsnorm(void* out, const void* in, const void* w, int64_t rows, int64_t dim, double eps,
                    int64_t in_stride, int64_t out_stride, int dt) {
  const size_t es = esize(dt);
  for (int64_t r = 0; r < rows; ++r) {
    rmsnorm_row((char*)out + r * out_stride * es, (const char*)in + r * in_stride * es, w, dim, eps, dt);
  }
}

/* Element-wise add (tests/kernel_tests.cu:206): a[i] + b[i] is a float sum. */
void oracle_add(void* out, const void* a, const void* b, int64_t n, int dt) {
  for (int64_t i = 0; i < n; ++i) stf(out, i, ldf(a, i, dt) + ldf(b, i, dt), dt);
}

static void add_rmsnorm_rows(void* h, const void* p, const void* w, void* y, int64_t r0, int64_t r1,
                             int64_t dim, double eps, int dt) {
  const size_t es = esize(dt);
  for (int64_t r = r0; r < r1; ++r) {
    void* hr = (char*)h + r * dim * es;
    oracle_add(hr, hr, (const char*)p + r * dim * es, dim, dt);
    rmsnorm_row((char*)y + r * dim * es, hr, w, dim, eps, dt);
  }
}

void oracle_add_rmsnorm(void* h, const void* p, const void* w, void* y, int64_t rows, int64_t dim, double eps,
                        int dt) {
  add_rmsnorm_rows(h, p, w, y, 0, rows, dim, eps, dt);
}

/* SwiGLU (tests/kernel_tests.cu:122): g / (1.0 + exp(-(double)g)) * up. */
void oracle_swiglu(void* out, const void* g, const void* u, int64_t n, int dt) {
  for (int64_t i = 0; i < n; ++i) {
    const double gv = ld(g, i, dt);
    st(out, i, gv / (1.0 + exp(-gv)) * ld(u, i, dt), dt);
  }
}

/* ------------------------------------------------------------------------- */
/* RoPE (tests/kernel_tests.cu:175-187, reference_rope):                      */
/*   angle = seq_pos / pow(theta, 2.0 * i / head_dim);                         */
/*   out[i] = first cos - second sin; out[i+half] = second cos + first sin.    */

static void rope_head(void* x, int64_t off, int pos, int hd, double theta, int dt, void* dst, int64_t dst_off) {
  const int half = hd / 2;
  for (int i = 0; i < half; ++i) {
    const double angle = pos / pow(theta, 2.0 * i / hd);
    const double first = ld(x, off + i, dt), second = ld(x, off + i + half, dt);
    const double c = cos(angle), s = sin(angle);
    st(dst, dst_off + i, first * c - second * s, dt);
    st(dst, dst_off + i + half, second * c + first * s, dt);
  }
}

void oracle_rope(void* x, const int32_t* positions, int32_t pos0, int64_t rows, int heads, int hd, double theta,
                 int dt) {
  for (int64_t r = 0; r < rows; ++r) {
    const int pos = positions ? positions[r] : (int)(pos0 + r);
    for (int h = 0; h < heads; ++h) {
      const int64_t off = (r * heads + h) * (int64_t)hd;
      rope_head(x, off, pos, hd, theta, dt, x, off);
    }
  }
}

/* KV store (tests/kernel_tests.cu:223-226):                                  */
/*   want[(h * max_seq + pos) * head_dim + d] = src[h * head_dim + d],         */
/* with a leading sequence dimension: cache [num_seqs][heads][max_seq][hd].    */
int32_t oracle_kv_store(void* cache, const void* src, const int32_t* positions, int32_t pos0,
                        const int32_t* seq_ids, int64_t rows, int heads, int hd, int max_seq, int num_seqs, int dt) {
  const size_t es = esize(dt);
  int32_t bad = 0;
  for (int64_t r = 0; r < rows; ++r) {
    const int pos = positions ? positions[r] : (int)(pos0 + r);
    const int seq = seq_ids ? seq_ids[r] : 0;
    int32_t b = 0;
    if (pos < 0 || pos >= max_seq) b |= BAD_POSITION;
    if (seq < 0 || seq >= num_seqs) b |= BAD_SEQUENCE;
    if (b) {
      bad |= b;
      continue;
    }
    for (int h = 0; h < heads; ++h) {
      const int64_t dst = (((int64_t)seq * heads + h) * max_seq + pos) * hd;
      memcpy((char*)cache + dst * es, (const char*)src + (r * heads + h) * (int64_t)hd * es, (size_t)hd * es);
    }
  }
  return bad;
}

static int32_t rope_kv_rows(void* q, const void* k, const void* v, const int32_t* positions, int32_t pos0,
                            const int32_t* seq_ids, void* k_cache, void* v_cache, int32_t table_len, double theta,
                            int64_t r0, int64_t r1, int hq, int hkv, int hd, int max_seq, int num_seqs, int dt) {
  const size_t es = esize(dt);
  int32_t bad = 0;
  for (int64_t r = r0; r < r1; ++r) {
    const int pos = positions ? positions[r] : (int)(pos0 + r);
    const int seq = seq_ids ? seq_ids[r] : 0;
    int32_t b = 0;
    if (pos < 0 || pos >= max_seq || (table_len > 0 && pos >= table_len)) b |= BAD_POSITION;
    if (seq < 0 || seq >= num_seqs) b |= BAD_SEQUENCE;
    if (b) {
      bad |= b;
      continue;
    }
    for (int h = 0; h < hq; ++h) {
      const int64_t off = (r * hq + h) * (int64_t)hd;
      rope_head(q, off, pos, hd, theta, dt, q, off);
    }
    for (int h = 0; h < hkv; ++h) {
      const int64_t src = (r * hkv + h) * (int64_t)hd;
      const int64_t dst = (((int64_t)seq * hkv + h) * max_seq + pos) * hd;
      rope_head((void*)k, src, pos, hd, theta, dt, k_cache, dst);
      memcpy((char*)v_cache + dst * es, (const char*)v + src * es, (size_t)hd * es);
    }
  }
  return bad;
}

/* q rotated in place; k rotated into k_cache (k unchanged); v copied into
 * v_cache. table_len > 0 also rejects positions >= table_len, as the kernel
 * does when it reads a table of that length. Returns BAD_* bits. */
int32_t oracle_rope_kv_store(void* q, const void* k, const void* v, const int32_t* positions, int32_t pos0,
                             const int32_t* seq_ids, void* k_cache, void* v_cache, int32_t table_len,
                             double theta, int64_t rows, int hq, int hkv, int hd, int max_seq, int num_seqs,
                             int dt) {
  return rope_kv_rows(q, k, v, positions, pos0, seq_ids, k_cache, v_cache, table_len, theta, 0, rows, hq, hkv,
                      hd, max_seq, num_seqs, dt);
}

/* (cos, sin) table [max_pos][hd/2] as fp32 pairs, from the same angle formula. */
void oracle_rope_table(float* table, int32_t max_pos, int hd, double theta) {
  const int half = hd / 2;
  for (int p = 0; p < max_pos; ++p) {
    for (int i = 0; i < half; ++i) {
      const double angle = p / pow(theta, 2.0 * i / hd);
      table[((int64_t)p * half + i) * 2 + 0] = (float)cos(angle);
      table[((int64_t)p * half + i) * 2 + 1] = (float)sin(angle);
    }
  }
}

/* Embedding gather: a row copy per token; ids outside [0, vocab) are skipped. */
static int32_t gather_rows(void* out, const void* table, const int32_t* ids, int64_t r0, int64_t r1, int64_t dim,
                           int64_t vocab, int64_t out_stride, int dt) {
  const size_t es = esize(dt);
  int32_t bad = 0;
  for (int64_t r = r0; r < r1; ++r) {
    const int32_t id = ids[r];
    if (id < 0 || id >= vocab) {
      bad |= BAD_ID;
      continue;
    }
    memcpy((char*)out + r * out_stride * es, (const char*)table + (int64_t)id * dim * es, (size_t)dim * es);
  }
  return bad;
}

int32_t oracle_gather(void* out, const void* table, const int32_t* ids, int64_t rows, int64_t dim, int64_t vocab,
                      int64_t out_stride, int dt) {
  return gather_rows(out, table, ids, 0, rows, dim, vocab, out_stride, dt);
}

/* ------------------------------------------------------------------------- */
/* One layer step over a row range: gather -> add+RMSNorm (attention norm) -> */
/* RoPE + KV store -> add+RMSNorm (FFN norm) -> SwiGLU. The CPU baseline.      */

typedef struct OracleStep {
  /* sizes */
  int64_t rows, dim, vocab, ffn;
  int32_t hq, hkv, hd, max_seq, num_seqs, table_len;
  double eps, theta;
  int32_t dtype;
  /* buffers (host) */
  const int32_t* ids;
  const void* embed;     /* [vocab][dim] */
  void* hidden;          /* [rows][dim]  gather output, residual */
  const void* attn_out;  /* [rows][dim]  delta of the first add */
  const void* w_attn;    /* [dim] */
  void* normed;          /* [rows][dim]  RMSNorm outputs */
  void* q;               /* [rows][hq][hd] */
  const void* k;         /* [rows][hkv][hd] */
  const void* v;         /* [rows][hkv][hd] */
  const int32_t* positions;
  const int32_t* seq_ids;
  void* k_cache;         /* [num_seqs][hkv][max_seq][hd] */
  void* v_cache;
  const void* ffn_out;   /* [rows][dim]  delta of the second add */
  const void* w_ffn;     /* [dim] */
  const void* gate;      /* [rows][ffn] */
  const void* up;        /* [rows][ffn] */
  void* act;             /* [rows][ffn] */
  int32_t ops;           /* bit mask of the ops to run: 1 gather, 2 attention add+RMSNorm, 4 RoPE+KV,
                            8 FFN add+RMSNorm, 16 SwiGLU (0 = all five) */
} OracleStep;

int32_t oracle_layer_step(const OracleStep* s, int64_t r0, int64_t r1) {
  const size_t es = esize(s->dtype);
  const int32_t ops = s->ops ? s->ops : 31;
  int32_t bad = 0;
  if (ops & 1) bad |= gather_rows(s->hidden, s->embed, s->ids, r0, r1, s->dim, s->vocab, s->dim, s->dtype);
  if (ops & 2) add_rmsnorm_rows(s->hidden, s->attn_out, s->w_attn, s->normed, r0, r1, s->dim, s->eps, s->dtype);
  if (ops & 4) {
    bad |= rope_kv_rows(s->q, s->k, s->v, s->positions, 0, s->seq_ids, s->k_cache, s->v_cache, s->table_len,
                        s->theta, r0, r1, s->hq, s->hkv, s->hd, s->max_seq, s->num_seqs, s->dtype);
  }
  if (ops & 8) add_rmsnorm_rows(s->hidden, s->ffn_out, s->w_ffn, s->normed, r0, r1, s->dim, s->eps, s->dtype);
  if (ops & 16) {
    oracle_swiglu((char*)s->act + r0 * s->ffn * es, (const char*)s->gate + r0 * s->ffn * es,
                  (const char*)s->up + r0 * s->ffn * es, (r1 - r0) * s->ffn, s->dtype);
  }
  return bad;
}

typedef struct {
  const OracleStep* s;
  int64_t r0, r1;
  int32_t bad;
} StepJob;

static void* step_worker(void* arg) {
  StepJob* j = (StepJob*)arg;
  j->bad = oracle_layer_step(j->s, j->r0, j->r1);
  return NULL;
}

/* Rows [r0, r1) split into `threads` contiguous blocks, one pthread each. */
int32_t oracle_layer_step_mt(const OracleStep* s, int64_t r0, int64_t r1, int threads) {
  if (threads <= 1 || r1 - r0 < 2) return oracle_layer_step(s, r0, r1);
  if (threads > 1024) threads = 1024;
  pthread_t* tid = (pthread_t*)calloc((size_t)threads, sizeof(pthread_t));
  StepJob* jobs = (StepJob*)calloc((size_t)threads, sizeof(StepJob));
  const int64_t n = r1 - r0;
  int started = 0;
  int32_t bad = 0;
  for (int t = 0; t < threads; ++t) {
    jobs[t].s = s;
    jobs[t].r0 = r0 + n * t / threads;
    jobs[t].r1 = r0 + n * (t + 1) / threads;
    if (jobs[t].r1 <= jobs[t].r0) continue;
    if (pthread_create(&tid[t], NULL, step_worker, &jobs[t]) != 0) {
      bad |= oracle_layer_step(s, jobs[t].r0, jobs[t].r1); /* run inline */
      jobs[t].r1 = jobs[t].r0;
      continue;
    }
    ++started;
  }
  for (int t = 0; t < threads; ++t) {
    if (jobs[t].r1 > jobs[t].r0) {
      pthread_join(tid[t], NULL);
      bad |= jobs[t].bad;
    }
  }
  (void)started;
  free(tid);
  free(jobs);
  return bad;
}

/* ------------------------------------------------------------------------- */
/* Decode attention (tests/kernel_tests.cu:229-258, test_attention):          */
/*   w[j] = exp(dot(q, k[j]) / sqrt(head_dim)), j < seq_len;                   */
/*   out[d] = sum_j w[j] / sum(w) * v[j][d],  all in double.                   */
/* Extended to a batch of queries: query b (num_q_heads heads) attends to      */
/* sequence seq_ids[b] of the cache [num_seqs][kv_heads][max_seq][head_dim]    */
/* over positions [0, lens[b]); q head h reads kv head h / (num_q_heads /      */
/* kv_heads) (GQA). The maximum score is subtracted before exp, which changes  */
/* nothing in exact arithmetic and keeps exp finite. Returns BAD_* bits; bad   */
/* queries leave their output untouched.                                        */
int32_t oracle_decode_attention(void* out, const void* q, const void* k_cache, const void* v_cache,
                                const int32_t* seq_ids, const int32_t* lens, int64_t batch, int hq, int hkv,
                                int hd, int max_seq, int num_seqs, int dt) {
  int32_t bad = 0;
  const int group = hkv > 0 ? hq / hkv : 1;
  double* w = (double*)malloc(sizeof(double) * (size_t)(max_seq > 0 ? max_seq : 1));
  double* acc = (double*)malloc(sizeof(double) * (size_t)hd);
  for (int64_t b = 0; b < batch; ++b) {
    const int seq = seq_ids ? seq_ids[b] : 0;
    const int len = lens[b];
    if (seq < 0 || seq >= num_seqs) {
      bad |= BAD_SEQUENCE;
      continue;
    }
    if (len <= 0 || len > max_seq) {
      bad |= BAD_POSITION;
      continue;
    }
    for (int h = 0; h < hq; ++h) {
      const int kvh = h / group;
      const int64_t qoff = (b * hq + h) * (int64_t)hd;
      const int64_t base = ((int64_t)seq * hkv + kvh) * max_seq * hd;
      double mx = -INFINITY, total = 0.0;
      for (int j = 0; j < len; ++j) {
        double dot = 0.0;
        for (int d = 0; d < hd; ++d) dot += ld(q, qoff + d, dt) * ld(k_cache, base + (int64_t)j * hd + d, dt);
        w[j] = dot / sqrt((double)hd);
        if (w[j] > mx) mx = w[j];
      }
      for (int j = 0; j < len; ++j) {
        w[j] = exp(w[j] - mx);
        total += w[j];
      }
      for (int d = 0; d < hd; ++d) acc[d] = 0.0;
      for (int j = 0; j < len; ++j) {
        const double p = w[j] / total;
        for (int d = 0; d < hd; ++d) acc[d] += p * ld(v_cache, base + (int64_t)j * hd + d, dt);
      }
      for (int d = 0; d < hd; ++d) st(out, qoff + d, acc[d], dt);
    }
  }
  free(w);
  free(acc);
  return bad;
}

/* ------------------------------------------------------------------------- */
/* GEMM (tests/kernel_tests.cu:49-59, reference_gemm; the product of           */
/* src/kernels.cu:83-113): c[row][col] = sum_i a[row][i] * b[i][col], the sum  */
/* in double over i = 0..k-1 in order, rounded once to the storage type.       */
/* a [m][k], b [k][n], c [m][n], all row-major.                                */
/* GEMM + SwiGLU (src/execution_engine.cu:122-124): gate and up are two such   */
/* sums (b = w_gate, w_up) and out = gate / (1 + exp(-gate)) * up in double    */
/* (the SwiGLU of tests/kernel_tests.cu:122), rounded once.                    */
/* Rows are split over `threads` pthreads; each works through blocks of 16     */
/* rows, widening each b row once per block.                                   */

typedef struct {
  void* c;
  const void* a;
  const void* b0;
  const void* b1; /* NULL: plain GEMM */
  int64_t r0, r1, n, k;
  int dt;
} GemmJob;

#define GEMM_ROW_BLOCK 16

static void gemm_rows(const GemmJob* j) {
  const int64_t n = j->n, k = j->k;
  const int sw = j->b1 != NULL;
  double* bg = (double*)malloc(sizeof(double) * (size_t)(n > 0 ? n : 1));
  double* bu = (double*)malloc(sizeof(double) * (size_t)(n > 0 ? n : 1));
  double* g = (double*)malloc(sizeof(double) * (size_t)(GEMM_ROW_BLOCK * (n > 0 ? n : 1)));
  double* u = (double*)malloc(sizeof(double) * (size_t)(GEMM_ROW_BLOCK * (n > 0 ? n : 1)));
  for (int64_t rb = j->r0; rb < j->r1; rb += GEMM_ROW_BLOCK) {
    const int64_t nr = (j->r1 - rb) < GEMM_ROW_BLOCK ? (j->r1 - rb) : GEMM_ROW_BLOCK;
    for (int64_t x = 0; x < nr * n; ++x) g[x] = u[x] = 0.0;
    for (int64_t i = 0; i < k; ++i) {
      for (int64_t col = 0; col < n; ++col) bg[col] = ld(j->b0, i * n + col, j->dt);
      if (sw) {
        for (int64_t col = 0; col < n; ++col) bu[col] = ld(j->b1, i * n + col, j->dt);
      }
      for (int64_t r = 0; r < nr; ++r) {
        const double av = ld(j->a, (rb + r) * k + i, j->dt);
        double* gr = g + r * n;
        for (int64_t col = 0; col < n; ++col) gr[col] += av * bg[col];
        if (sw) {
          double* ur = u + r * n;
          for (int64_t col = 0; col < n; ++col) ur[col] += av * bu[col];
        }
      }
    }
    for (int64_t r = 0; r < nr; ++r) {
      for (int64_t col = 0; col < n; ++col) {
        const double gv = g[r * n + col];
        const double v = sw ? gv / (1.0 + exp(-gv)) * u[r * n + col] : gv;
        st(j->c, (rb + r) * n + col, v, j->dt);
      }
    }
  }
  free(bg);
  free(bu);
  free(g);
  free(u);
}

static void* gemm_worker(void* arg) {
  gemm_rows((const GemmJob*)arg);
  return NULL;
}

static void gemm_mt(void* c, const void* a, const void* b0, const void* b1, int64_t m, int64_t n, int64_t k,
                    int dt, int threads) {
  if (threads < 1) threads = 1;
  if (threads > m) threads = m > 0 ? (int)m : 1;
  GemmJob* jobs = (GemmJob*)calloc((size_t)threads, sizeof(GemmJob));
  pthread_t* tid = (pthread_t*)calloc((size_t)threads, sizeof(pthread_t));
  int* started = (int*)calloc((size_t)threads, sizeof(int));
  for (int t = 0; t < threads; ++t) {
    jobs[t].c = c;
    jobs[t].a = a;
    jobs[t].b0 = b0;
    jobs[t].b1 = b1;
    jobs[t].r0 = m * t / threads;
    jobs[t].r1 = m * (t + 1) / threads;
    jobs[t].n = n;
    jobs[t].k = k;
    jobs[t].dt = dt;
    if (t > 0) started[t] = pthread_create(&tid[t], NULL, gemm_worker, &jobs[t]) == 0;
  }
  gemm_rows(&jobs[0]);
  for (int t = 1; t < threads; ++t) {
    if (started[t]) {
      pthread_join(tid[t], NULL);
    } else {
      gemm_rows(&jobs[t]); /* no thread: run its rows here */
    }
  }
  free(started);
  free(tid);
  free(jobs);
}

void oracle_gemm(void* c, const void* a, const void* b, int64_t m, int64_t n, int64_t k, int dt, int threads) {
  gemm_mt(c, a, b, NULL, m, n, k, dt, threads);
}

void oracle_gemm_swiglu(void* out, const void* x, const void* w_gate, const void* w_up, int64_t rows, int64_t dim,
                        int64_t hidden, int dt, int threads) {
  gemm_mt(out, x, w_gate, w_up, rows, hidden, dim, dt, threads);
}

/* ------------------------------------------------------------------------- */
/* Softmax in place (tests/kernel_tests.cu:105-160): for each of num_vectors   */
/* vectors of `size` elements, `stride` apart, x = exp(x - max) / sum exp(x -   */
/* max) with the sum in double, rounded once; the gaps are left untouched.      */
void oracle_softmax(void* x, int64_t size, int64_t num_vectors, int64_t stride, int dt) {
  for (int64_t v = 0; v < num_vectors; ++v) {
    const int64_t off = v * stride;
    double mx = -INFINITY, total = 0.0;
    for (int64_t i = 0; i < size; ++i) {
      const double e = ld(x, off + i, dt);
      if (e > mx) mx = e;
    }
    for (int64_t i = 0; i < size; ++i) total += exp(ld(x, off + i, dt) - mx);
    for (int64_t i = 0; i < size; ++i) st(x, off + i, exp(ld(x, off + i, dt) - mx) / total, dt);
  }
}
