/*
 * fgt_oracle.c — TEST INFRASTRUCTURE ONLY: a CPU restatement of the
 * reference's semantics for fused elementwise / broadcast / reduction
 * partitions, used as the parity checker and as the timed CPU baseline.
 * Nothing in the product (fugatensor_b200/) links, imports or calls it.
 *
 * The reference evaluates these partitions through the external ASK SDK
 * 0.1.0 (CMakeLists.txt:15), which is not in the reference tree; its CPU JIT
 * (src/fugatensor/backends/host.py:239-264) cannot be built or run here.
 * This file restates the semantics the reference's own tests pin, per op:
 *   - every IR-visible op rounds to its result dtype; f16/bf16 arithmetic is
 *     f32 arithmetic rounded once (RNE, subnormals, overflow -> inf)
 *     (src/fugatensor/_ask/numerics.py:28-78, tests/backend/support/pointwise.py:147-200);
 *   - no FMA contraction (tests/backend/test_host_compiler.py:127-138);
 *   - casts: float->int saturating with NaN -> 0 and truncation, x->bool is
 *     x != 0 (tests/backend/support/pointwise.py:239-253);
 *   - integer arithmetic wraps; floordiv/mod/shift per tests/support/stage2.py:36-67;
 *   - reduce_max/min are IEEE: NaN propagates, +0 beats -0 for max
 *     (tests/support/reduction_max.py:64-70);
 *   - argmax/argmin: first occurrence, NaN counts as the extremum, i64
 *     (tests/test_stage2_ops.py:148-157, src/fugatensor/ir/tensor_rules.py:95-108);
 *   - reduce_sum in mode LITERAL accumulates left to right in the storage
 *     dtype (tests/test_tensor_primitives.py:184-192); in mode ACCURATE it
 *     accumulates in f64 and rounds once (the definition used to check the
 *     large configurations, where the literal order is not pinned).
 * Transcendentals use the C library's f32 functions (expf, logf, ...).
 */
#include <float.h>
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "../include/fgt.h"

#define MODE_LITERAL 0
#define MODE_ACCURATE 1

typedef struct {
  int dt;
  int rank;
  int64_t shape[FGT_MAX_RANK];
  int64_t n;
  void* v; /* bool: uint8, i32: int32, i64: int64, floats: float (exact value) */
} Buf;

static int is_float(int dt) { return dt == FGT_F32 || dt == FGT_F16 || dt == FGT_BF16; }
static size_t vsize(int dt) {
  switch (dt) {
    case FGT_BOOL: return 1;
    case FGT_I32: return 4;
    case FGT_I64: return 8;
    default: return 4;
  }
}

/* ------------------------------------------------------------ rounding -- */
/* Round an exact long double (64-bit significand) once to a binary format
 * with p significand bits and minimum normal exponent emin; RNE. */
static float round_format(long double x, int p, int emin, long double maxv) {
  if (x != x || x == 0 || isinf(x)) return (float)x;
  int e = ilogbl(x);
  if (e < emin) e = emin;
  long double q = ldexpl(x, p - 1 - e);
  q = nearbyintl(q);
  long double r = ldexpl(q, e - (p - 1));
  if (fabsl(r) > maxv) return x < 0 ? -INFINITY : INFINITY;
  return (float)r;
}
static float rnd_dt(long double x, int dt) {
  switch (dt) {
    case FGT_F16: return round_format(x, 11, -14, 65504.0L);
    case FGT_BF16: return round_format(x, 8, -126, ldexpl(255.0L, 120));
    default: return round_format(x, 24, -126, (long double)FLT_MAX);
  }
}
/* Fast paths for a value that is already an f32: f32 is the identity; bf16
 * shares f32's exponent range, so RNE on the bit pattern is exact (overflow
 * carries into the exponent and yields inf); f16 scales to an integer
 * significand (exact power-of-two scaling) and rounds with nearbyintf (RNE). */
static float rnd_bf16_f(float x) {
  uint32_t u;
  memcpy(&u, &x, 4);
  if ((u & 0x7f800000u) == 0x7f800000u) {
    if (u & 0x7fffffu) u |= 0x400000u;
    memcpy(&x, &u, 4);
    return x;
  }
  u += 0x7fffu + ((u >> 16) & 1u);
  u &= 0xffff0000u;
  memcpy(&x, &u, 4);
  return x;
}
static float rnd_f16_f(float x) {
  if (x != x || isinf(x) || x == 0) return x;
  float a = fabsf(x);
  int e = ilogbf(a);
  if (e < -14) e = -14;
  float q = ldexpf(nearbyintf(ldexpf(a, 10 - e)), e - 10);
  if (q > 65504.0f) q = INFINITY;
  return x < 0 ? -q : q;
}
static float rnd_f(float x, int dt) {
  if (dt == FGT_F16) return rnd_f16_f(x);
  if (dt == FGT_BF16) return rnd_bf16_f(x);
  return x;
}

static float f16_decode(uint16_t h) {
  int s = h >> 15, e = (h >> 10) & 31, f = h & 1023;
  float v;
  if (e == 31) v = f ? NAN : INFINITY;
  else if (e == 0) v = ldexpf((float)f, -24);
  else v = ldexpf((float)(f | 1024), e - 25);
  return s ? -v : v;
}
static uint16_t f16_encode(float x) { /* x already exactly representable */
  uint32_t u;
  memcpy(&u, &x, 4);
  uint16_t s = (uint16_t)((u >> 16) & 0x8000);
  if (x != x) return s | 0x7e00;
  float a = fabsf(x);
  if (isinf(a)) return s | 0x7c00;
  if (a == 0) return s;
  int e = ilogbf(a);
  if (e < -14) return s | (uint16_t)lrintf(ldexpf(a, 24));
  uint16_t frac = (uint16_t)lrintf(ldexpf(a, 10 - e)) & 1023;
  return s | (uint16_t)((e + 15) << 10) | frac;
}
static float bf16_decode(uint16_t h) {
  uint32_t u = (uint32_t)h << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}
static uint16_t bf16_encode(float x) {
  uint32_t u;
  memcpy(&u, &x, 4);
  if (x != x) return (uint16_t)((u >> 16) | 0x40);
  return (uint16_t)(u >> 16);
}

/* ----------------------------------------------------------- helpers ----- */
static int64_t numel(const int64_t* s, int r) {
  int64_t n = 1;
  for (int i = 0; i < r; ++i) n *= s[i];
  return n;
}
static void strides(const int64_t* s, int r, int64_t* st) {
  int64_t a = 1;
  for (int i = r - 1; i >= 0; --i) {
    st[i] = a;
    a *= s[i];
  }
}
static void unravel(int64_t lin, const int64_t* s, int r, int64_t* c) {
  for (int i = r - 1; i >= 0; --i) {
    if (s[i]) {
      c[i] = lin % s[i];
      lin /= s[i];
    } else c[i] = 0;
  }
}

/* value access as long double (numeric) */
static long double getf(const Buf* b, int64_t i) {
  switch (b->dt) {
    case FGT_BOOL: return ((uint8_t*)b->v)[i];
    case FGT_I32: return ((int32_t*)b->v)[i];
    case FGT_I64: return ((int64_t*)b->v)[i];
    default: return ((float*)b->v)[i];
  }
}
static int64_t geti(const Buf* b, int64_t i) {
  switch (b->dt) {
    case FGT_BOOL: return ((uint8_t*)b->v)[i];
    case FGT_I32: return ((int32_t*)b->v)[i];
    default: return ((int64_t*)b->v)[i];
  }
}

static float fmax_ieee(float a, float b) {
  if (a != a) return a;
  if (b != b) return b;
  if (a == b) return signbit(a) ? b : a;
  return a > b ? a : b;
}
static float fmin_ieee(float a, float b) {
  if (a != a) return a;
  if (b != b) return b;
  if (a == b) return signbit(a) ? a : b;
  return a < b ? a : b;
}

static int64_t wrap(int64_t v, int dt) { return dt == FGT_I32 ? (int64_t)(int32_t)(uint32_t)(uint64_t)v : v; }
static int64_t iminv(int dt) { return dt == FGT_I32 ? INT32_MIN : INT64_MIN; }
static int bits_of(int dt) { return dt == FGT_I32 ? 32 : 64; }

static int64_t ifloordiv(int64_t a, int64_t b, int dt) {
  if (b == 0) return 0;
  if (a == iminv(dt) && b == -1) return iminv(dt);
  int64_t q = a / b;
  if ((a % b != 0) && ((a < 0) != (b < 0))) q -= 1;
  return q;
}
static int64_t imod(int64_t a, int64_t b, int dt) {
  if (b == 0) return 0;
  if (a == iminv(dt) && b == -1) return 0;
  int64_t r = a % b;
  if (r != 0 && ((r < 0) != (b < 0))) r += b;
  return r;
}
static int64_t ipow(int64_t base, int64_t e, int dt) {
  if (e < 0) {
    if (base == 1) return 1;
    if (base == -1) return (e & 1) ? -1 : 1;
    return 0;
  }
  uint64_t r = 1, b = (uint64_t)base;
  while (e) {
    if (e & 1) r *= b;
    b *= b;
    e >>= 1;
  }
  return wrap((int64_t)r, dt);
}

static void seterr(char* err, size_t cap, const char* m) {
  if (err && cap) snprintf(err, cap, "%s", m);
}

/* --------------------------------------------------------------- eval ---- */
static float f_unary(int op, float a) {
  switch (op) {
    case FGT_OP_EXP: return expf(a);
    case FGT_OP_LOG: return logf(a);
    case FGT_OP_SQRT: return sqrtf(a);
    case FGT_OP_SIN: return sinf(a);
    case FGT_OP_COS: return cosf(a);
    case FGT_OP_TANH: return tanhf(a);
    case FGT_OP_ERF: return erff(a);
    case FGT_OP_ABS: return fabsf(a);
    case FGT_OP_FLOOR: return floorf(a);
    case FGT_OP_CEIL: return ceilf(a);
    case FGT_OP_ROUND: return nearbyintf(a);
  }
  return NAN;
}
static float f_binary(int op, float a, float b) {
  switch (op) {
    case FGT_OP_ADD: return a + b;
    case FGT_OP_MUL: return a * b;
    case FGT_OP_DIV: return a / b;
    case FGT_OP_MAXIMUM: return fmax_ieee(a, b);
    case FGT_OP_MINIMUM: return fmin_ieee(a, b);
    case FGT_OP_POW: return powf(a, b);
    case FGT_OP_FLOORDIV: return floorf(a / b);
    case FGT_OP_MOD: {
      float r = fmodf(a, b);
      if (r != 0.0f && ((r < 0.0f) != (b < 0.0f))) r = r + b;
      return r;
    }
  }
  return NAN;
}
static int64_t i_binary(int op, int64_t a, int64_t b, int dt) {
  switch (op) {
    case FGT_OP_ADD: return wrap((int64_t)((uint64_t)a + (uint64_t)b), dt);
    case FGT_OP_MUL: return wrap((int64_t)((uint64_t)a * (uint64_t)b), dt);
    case FGT_OP_MAXIMUM: return a > b ? a : b;
    case FGT_OP_MINIMUM: return a < b ? a : b;
    case FGT_OP_POW: return ipow(a, b, dt);
    case FGT_OP_FLOORDIV: return ifloordiv(a, b, dt);
    case FGT_OP_MOD: return imod(a, b, dt);
    case FGT_OP_BITWISE_AND: return a & b;
    case FGT_OP_BITWISE_OR: return a | b;
    case FGT_OP_BITWISE_XOR: return a ^ b;
    case FGT_OP_SHIFT_LEFT:
      if (b < 0 || b >= bits_of(dt)) return 0;
      return wrap((int64_t)((uint64_t)a << b), dt);
    case FGT_OP_SHIFT_RIGHT:
      if (b < 0) return 0;
      if (b >= bits_of(dt)) return a < 0 ? -1 : 0;
      return a >> b;
  }
  return 0;
}

/* store a numeric value (already of the node's semantics) into buffer */
static void put_int(Buf* b, int64_t i, int64_t v) {
  switch (b->dt) {
    case FGT_BOOL: ((uint8_t*)b->v)[i] = v != 0; break;
    case FGT_I32: ((int32_t*)b->v)[i] = (int32_t)v; break;
    default: ((int64_t*)b->v)[i] = v; break;
  }
}

static void cast_one(const Buf* x, int64_t i, Buf* o, int64_t j) {
  int from = x->dt, to = o->dt;
  if (to == FGT_BOOL) {
    ((uint8_t*)o->v)[j] = is_float(from) ? (((float*)x->v)[i] != 0.0f) : (geti(x, i) != 0);
    return;
  }
  if (is_float(to)) {
    /* a float source is an exact f32 value: the f32-input rounding is exact */
    if (is_float(from)) ((float*)o->v)[j] = rnd_f(((float*)x->v)[i], to);
    else ((float*)o->v)[j] = rnd_dt((long double)geti(x, i), to);
    return;
  }
  if (is_float(from)) {
    float f = ((float*)x->v)[i];
    int64_t lo = iminv(to), hi = to == FGT_I32 ? INT32_MAX : INT64_MAX;
    int64_t r;
    if (f != f) r = 0;
    else if (f <= (long double)lo) r = lo;
    else if (f >= (long double)hi) r = hi;
    else r = (int64_t)truncf(f);
    put_int(o, j, r);
    return;
  }
  put_int(o, j, wrap(geti(x, i), to));
}

static int arg_better(int is_max, int fl, long double a, int64_t ia, long double b, int64_t ib) {
  if (fl) {
    int an = a != a, bn = b != b;
    if (an || bn) return (an && bn) ? ia < ib : an;
  }
  if (is_max ? a > b : a < b) return 1;
  if (is_max ? a < b : a > b) return 0;
  return ia < ib;
}

/* Partial state of one reduction over a range of its reduced elements. */
typedef struct {
  long double accd;
  float accf;
  int64_t acci;
  int have;
  long double best;
  int64_t besti;
  float mf;
  int64_t mi;
  int bacc;
} RedPart;

typedef struct {
  const fgt_node* nd;
  const Buf* x;
  int mode, fl, nr, trailing;
  int isred[FGT_MAX_RANK];
  int64_t xs[FGT_MAX_RANK], red[FGT_MAX_RANK], rstride0;
} RedCtx;

static void red_init(const RedCtx* c, RedPart* p) {
  const int op = c->nd->opcode;
  p->accd = op == FGT_OP_REDUCE_PROD ? 1.0L : 0.0L;
  p->accf = op == FGT_OP_REDUCE_PROD ? 1.0f : 0.0f;
  p->acci = op == FGT_OP_REDUCE_PROD ? 1 : 0;
  p->have = 0;
  p->best = 0;
  p->besti = 0;
  p->mf = 0;
  p->mi = 0;
  p->bacc = op == FGT_OP_REDUCE_ALL ? 1 : 0;
}

/* Offset of reduced element ri (row-major over the reduced axes) from the
 * kept coordinates' base. One reduced axis and trailing contiguous reduced
 * axes (every benchmark partition) take the direct forms. */
static int64_t red_off(const RedCtx* c, int64_t base, int64_t ri) {
  if (c->nr == 1) return base + ri * c->rstride0;
  if (c->trailing) return base + ri;
  int64_t rc[FGT_MAX_RANK];
  unravel(ri, c->red, c->nr, rc);
  int64_t off = base;
  int t = 0;
  for (int k = 0; k < c->x->rank; ++k)
    if (c->isred[k]) off += rc[t++] * c->xs[k];
  return off;
}

/* Fold reduced elements [lo, hi) into p, left to right. */
static void red_range(const RedCtx* c, int64_t base, int64_t lo, int64_t hi, RedPart* p) {
  const int op = c->nd->opcode, fl = c->fl, mode = c->mode;
  const Buf* x = c->x;
  for (int64_t ri = lo; ri < hi; ++ri) {
    const int64_t off = red_off(c, base, ri);
    switch (op) {
      case FGT_OP_REDUCE_SUM:
      case FGT_OP_REDUCE_PROD:
        if (fl) {
          float v = ((float*)x->v)[off];
          if (mode == MODE_ACCURATE)
            p->accd = op == FGT_OP_REDUCE_SUM ? p->accd + (double)v : (long double)((double)p->accd * (double)v);
          else p->accf = rnd_f(op == FGT_OP_REDUCE_SUM ? p->accf + v : p->accf * v, x->dt);
        } else {
          int64_t v = geti(x, off);
          p->acci = wrap(op == FGT_OP_REDUCE_SUM ? (int64_t)((uint64_t)p->acci + (uint64_t)v)
                                                 : (int64_t)((uint64_t)p->acci * (uint64_t)v), x->dt);
        }
        break;
      case FGT_OP_REDUCE_MAX:
      case FGT_OP_REDUCE_MIN:
        if (fl) {
          float v = ((float*)x->v)[off];
          p->mf = !p->have ? v : (op == FGT_OP_REDUCE_MAX ? fmax_ieee(p->mf, v) : fmin_ieee(p->mf, v));
        } else {
          int64_t v = geti(x, off);
          p->mi = !p->have ? v : (op == FGT_OP_REDUCE_MAX ? (v > p->mi ? v : p->mi) : (v < p->mi ? v : p->mi));
        }
        p->have = 1;
        break;
      case FGT_OP_REDUCE_ANY: p->bacc = p->bacc || ((uint8_t*)x->v)[off]; break;
      case FGT_OP_REDUCE_ALL: p->bacc = p->bacc && ((uint8_t*)x->v)[off]; break;
      case FGT_OP_ARGMAX:
      case FGT_OP_ARGMIN: {
        /* one reduced axis: the index along it is ri */
        long double v = getf(x, off);
        if (!p->have || arg_better(op == FGT_OP_ARGMAX, fl, v, ri, p->best, p->besti)) {
          p->best = v;
          p->besti = ri;
        }
        p->have = 1;
        break;
      }
    }
  }
}

/* p <- p followed by q (q covers the elements after p's). Only for the
 * reductions red_splittable() admits, where this equals one left-to-right
 * fold up to the rounding of the long double sum. */
static void red_merge(const RedCtx* c, RedPart* p, const RedPart* q) {
  const int op = c->nd->opcode, fl = c->fl;
  switch (op) {
    case FGT_OP_REDUCE_SUM:
      if (fl) p->accd = p->accd + q->accd;
      else p->acci = wrap((int64_t)((uint64_t)p->acci + (uint64_t)q->acci), c->x->dt);
      break;
    case FGT_OP_REDUCE_PROD: p->acci = wrap((int64_t)((uint64_t)p->acci * (uint64_t)q->acci), c->x->dt); break;
    case FGT_OP_REDUCE_MAX:
    case FGT_OP_REDUCE_MIN:
      if (!q->have) break;
      if (!p->have) {
        p->mf = q->mf;
        p->mi = q->mi;
      } else if (fl) p->mf = op == FGT_OP_REDUCE_MAX ? fmax_ieee(p->mf, q->mf) : fmin_ieee(p->mf, q->mf);
      else p->mi = op == FGT_OP_REDUCE_MAX ? (q->mi > p->mi ? q->mi : p->mi) : (q->mi < p->mi ? q->mi : p->mi);
      p->have = 1;
      break;
    case FGT_OP_REDUCE_ANY: p->bacc = p->bacc || q->bacc; break;
    case FGT_OP_REDUCE_ALL: p->bacc = p->bacc && q->bacc; break;
    case FGT_OP_ARGMAX:
    case FGT_OP_ARGMIN:
      if (q->have && (!p->have || arg_better(op == FGT_OP_ARGMAX, fl, q->best, q->besti, p->best, p->besti))) {
        p->best = q->best;
        p->besti = q->besti;
      }
      p->have = p->have || q->have;
      break;
  }
}

/* Reductions whose result does not depend on how the range is split:
 * integer sums/products (wrapping arithmetic is associative), max/min,
 * arg-reductions (index tie-break), any/all, and ACCURATE float sums (long
 * double partials; the split changes only bits far below the f64 result that
 * is rounded once). LITERAL float sums fix a left-to-right order and float
 * products a double-rounding order, so they stay sequential. */
static int red_splittable(const RedCtx* c) {
  const int op = c->nd->opcode;
  if (op == FGT_OP_REDUCE_PROD) return !c->fl;
  if (op == FGT_OP_REDUCE_SUM) return !c->fl || c->mode == MODE_ACCURATE;
  return 1;
}

#define RED_CHUNK ((int64_t)1 << 20)
/* loops over fewer elements than this run on the calling thread */
#define PAR_MIN ((int64_t)1 << 15)

static int eval_reduce(const fgt_node* nd, const Buf* x, Buf* o, int mode, int threads) {
  RedCtx c;
  memset(&c, 0, sizeof c);
  c.nd = nd;
  c.x = x;
  c.mode = mode;
  c.fl = is_float(x->dt);
  int axes[FGT_MAX_RANK] = {0};
  int nax = 0;
  if (nd->opcode == FGT_OP_ARGMAX || nd->opcode == FGT_OP_ARGMIN) {
    axes[0] = (int)nd->attrs[0];
    nax = 1;
  } else {
    for (int k = 0; k < nd->num_attrs; ++k) axes[nax++] = (int)nd->attrs[k];
  }
  for (int k = 0; k < nax; ++k) c.isred[axes[k]] = 1;
  strides(x->shape, x->rank, c.xs);
  int64_t kept[FGT_MAX_RANK];
  int nk = 0;
  for (int k = 0; k < x->rank; ++k) {
    if (c.isred[k]) {
      if (c.nr == 0) c.rstride0 = c.xs[k];
      c.red[c.nr++] = x->shape[k];
    } else kept[nk++] = x->shape[k];
  }
  c.trailing = 1;
  for (int k = x->rank - c.nr; k < x->rank; ++k)
    if (k < 0 || !c.isred[k]) c.trailing = 0;
  const int64_t nred = numel(c.red, c.nr);
  const int op = nd->opcode;
  const int64_t nchunks = (nred + RED_CHUNK - 1) / RED_CHUNK;
  /* one output over a long range (a whole-tensor reduction): split the range
   * into fixed chunks, folded in parallel and merged in order (the result does
   * not depend on the thread count); otherwise one output per iteration */
  const int split = red_splittable(&c) && nchunks > 1 && o->n == 1;
  RedPart whole;
  red_init(&c, &whole);
  if (split) {
    RedPart* parts = (RedPart*)malloc(sizeof(RedPart) * (size_t)nchunks);
    if (!parts) return 1;
#pragma omp parallel for num_threads(threads) schedule(dynamic, 1)
    for (int64_t q = 0; q < nchunks; ++q) {
      red_init(&c, &parts[q]);
      const int64_t hi = (q + 1) * RED_CHUNK < nred ? (q + 1) * RED_CHUNK : nred;
      red_range(&c, 0, q * RED_CHUNK, hi, &parts[q]);
    }
    for (int64_t q = 1; q < nchunks; ++q) red_merge(&c, &parts[0], &parts[q]);
    whole = parts[0];
    free(parts);
  }
#pragma omp parallel for num_threads(threads) schedule(static) if (!split && o->n > 1)
  for (int64_t oi = 0; oi < o->n; ++oi) {
    RedPart p;
    if (split) {
      p = whole;
    } else {
      int64_t oc[FGT_MAX_RANK];
      unravel(oi, kept, nk, oc);
      int64_t base = 0;
      int t = 0;
      for (int k = 0; k < x->rank; ++k)
        if (!c.isred[k]) base += oc[t++] * c.xs[k];
      red_init(&c, &p);
      red_range(&c, base, 0, nred, &p);
    }
    switch (op) {
      case FGT_OP_REDUCE_SUM:
      case FGT_OP_REDUCE_PROD:
        if (c.fl) ((float*)o->v)[oi] = mode == MODE_ACCURATE ? rnd_dt((long double)(double)p.accd, x->dt) : p.accf;
        else put_int(o, oi, p.acci);
        break;
      case FGT_OP_REDUCE_MAX:
      case FGT_OP_REDUCE_MIN:
        if (c.fl) ((float*)o->v)[oi] = p.mf;
        else put_int(o, oi, p.mi);
        break;
      case FGT_OP_REDUCE_ANY:
      case FGT_OP_REDUCE_ALL: ((uint8_t*)o->v)[oi] = (uint8_t)p.bacc; break;
      default: ((int64_t*)o->v)[oi] = p.besti; break;
    }
  }
  return 0;
}

static void load_input(Buf* b, const void* src, int threads) {
#pragma omp parallel for num_threads(threads) schedule(static) if (b->n >= PAR_MIN)
  for (int64_t i = 0; i < b->n; ++i) {
    switch (b->dt) {
      case FGT_BOOL: ((uint8_t*)b->v)[i] = ((const uint8_t*)src)[i] != 0; break;
      case FGT_I32: ((int32_t*)b->v)[i] = ((const int32_t*)src)[i]; break;
      case FGT_I64: ((int64_t*)b->v)[i] = ((const int64_t*)src)[i]; break;
      case FGT_F32: ((float*)b->v)[i] = ((const float*)src)[i]; break;
      case FGT_F16: ((float*)b->v)[i] = f16_decode(((const uint16_t*)src)[i]); break;
      case FGT_BF16: ((float*)b->v)[i] = bf16_decode(((const uint16_t*)src)[i]); break;
    }
  }
}
static void store_output(const Buf* b, void* dst, int threads) {
#pragma omp parallel for num_threads(threads) schedule(static) if (b->n >= PAR_MIN)
  for (int64_t i = 0; i < b->n; ++i) {
    switch (b->dt) {
      case FGT_BOOL: ((uint8_t*)dst)[i] = ((uint8_t*)b->v)[i]; break;
      case FGT_I32: ((int32_t*)dst)[i] = ((int32_t*)b->v)[i]; break;
      case FGT_I64: ((int64_t*)dst)[i] = ((int64_t*)b->v)[i]; break;
      case FGT_F32: ((float*)dst)[i] = ((float*)b->v)[i]; break;
      case FGT_F16: ((uint16_t*)dst)[i] = f16_encode(((float*)b->v)[i]); break;
      case FGT_BF16: ((uint16_t*)dst)[i] = bf16_encode(((float*)b->v)[i]); break;
    }
  }
}

static float const_value_f(int dt, uint64_t bits) {
  if (dt == FGT_F32) {
    uint32_t u = (uint32_t)bits;
    float f;
    memcpy(&f, &u, 4);
    return f;
  }
  if (dt == FGT_F16) return f16_decode((uint16_t)bits);
  return bf16_decode((uint16_t)bits);
}

/* o[j] = a[off(j)] with off(j) = sum_k coord_k(j) * step[k]: one unravel per
 * run of the innermost output axis, then a strided walk. */
static void gather_runs(const Buf* a, Buf* o, const int64_t* step, int threads) {
  const int r = o->rank;
  const int64_t inner = r ? o->shape[r - 1] : 1;
  const int64_t runs = inner ? o->n / inner : 0;
  const int64_t istep = r ? step[r - 1] : 0;
  const size_t w = vsize(o->dt);
#pragma omp parallel for num_threads(threads) schedule(static) if (o->n >= PAR_MIN)
  for (int64_t q = 0; q < runs; ++q) {
    int64_t cc[FGT_MAX_RANK];
    unravel(q * inner, o->shape, r, cc);
    int64_t off = 0;
    for (int k = 0; k + 1 < r; ++k) off += cc[k] * step[k];
    char* dst = (char*)o->v + (size_t)(q * inner) * w;
    const char* src = (const char*)a->v;
    if (w == 4) {
      for (int64_t i = 0; i < inner; ++i) ((uint32_t*)dst)[i] = ((const uint32_t*)src)[off + i * istep];
    } else if (w == 8) {
      for (int64_t i = 0; i < inner; ++i) ((uint64_t*)dst)[i] = ((const uint64_t*)src)[off + i * istep];
    } else {
      for (int64_t i = 0; i < inner; ++i) dst[i] = src[off + i * istep];
    }
  }
}

/* Evaluate a partition: mode 0 literal, 1 accurate, on `threads` threads
 * (every result is independent of the thread count). Returns 0 on success. */
static int eval_impl(const fgt_partition_desc* d, int mode, const void* const* inputs, void* const* outputs, char* err,
                     size_t errcap, int threads) {
  if (threads < 1) threads = 1;
  const int N = d->num_nodes;
  Buf* B = (Buf*)calloc((size_t)N, sizeof(Buf));
  int* last = (int*)malloc(sizeof(int) * (size_t)N);
  if (!B || !last) {
    seterr(err, errcap, "out of memory");
    return 1;
  }
  for (int i = 0; i < N; ++i) last[i] = i;
  for (int i = 0; i < N; ++i)
    for (int k = 0; k < d->nodes[i].num_operands; ++k) last[d->nodes[i].operands[k]] = i;
  for (int k = 0; k < d->num_outputs; ++k) last[d->outputs[k]] = N;
  int rc = 0;
  for (int i = 0; i < N && !rc; ++i) {
    const fgt_node* nd = &d->nodes[i];
    Buf* o = &B[i];
    o->dt = nd->dtype;
    o->rank = nd->rank;
    for (int k = 0; k < nd->rank; ++k) o->shape[k] = nd->shape[k];
    o->n = numel(o->shape, o->rank);
    o->v = malloc((size_t)(o->n ? o->n : 1) * vsize(o->dt));
    if (!o->v) {
      seterr(err, errcap, "out of memory");
      rc = 1;
      break;
    }
    const Buf* a = nd->num_operands > 0 ? &B[nd->operands[0]] : NULL;
    const Buf* b = nd->num_operands > 1 ? &B[nd->operands[1]] : NULL;
    const Buf* c = nd->num_operands > 2 ? &B[nd->operands[2]] : NULL;
    const int op = nd->opcode;
    int64_t os[FGT_MAX_RANK], as[FGT_MAX_RANK], cc[FGT_MAX_RANK], xc[FGT_MAX_RANK];
    strides(o->shape, o->rank, os);
    switch (op) {
      case FGT_OP_PARAMETER: load_input(o, inputs[nd->attrs[0]], threads); break;
      case FGT_OP_CONSTANT:
        if (is_float(o->dt)) ((float*)o->v)[0] = const_value_f(o->dt, nd->constant_bits);
        else if (o->dt == FGT_I32) ((int32_t*)o->v)[0] = (int32_t)(uint32_t)nd->constant_bits;
        else if (o->dt == FGT_I64) ((int64_t*)o->v)[0] = (int64_t)nd->constant_bits;
        else ((uint8_t*)o->v)[0] = (nd->constant_bits & 0xff) != 0;
        break;
      case FGT_OP_SPLAT:
#pragma omp parallel for num_threads(threads) schedule(static) if (o->n >= PAR_MIN)
        for (int64_t j = 0; j < o->n; ++j) memcpy((char*)o->v + j * vsize(o->dt), a->v, vsize(o->dt));
        break;
      case FGT_OP_RESHAPE:
      case FGT_OP_STOP_GRADIENT: memcpy(o->v, a->v, (size_t)o->n * vsize(o->dt)); break;
      case FGT_OP_BROADCAST_IN_DIM:
      case FGT_OP_TRANSPOSE: {
        /* output element j reads operand offset sum_k coord_k * step_k, where
         * step_k is the operand stride that output axis k moves (0 for an
         * expanded axis); walked one innermost run at a time */
        strides(a->shape, a->rank, as);
        int64_t step[FGT_MAX_RANK] = {0};
        if (op == FGT_OP_TRANSPOSE) {
          for (int k = 0; k < o->rank; ++k) step[k] = as[nd->attrs[k]];
        } else {
          for (int k = 0; k < a->rank; ++k)
            if (a->shape[k] != 1) step[nd->attrs[k]] += as[k];
        }
        gather_runs(a, o, step, threads);
        break;
      }
      case FGT_OP_IOTA:
#pragma omp parallel for num_threads(threads) schedule(static) if (o->n >= PAR_MIN) private(cc)
        for (int64_t j = 0; j < o->n; ++j) {
          unravel(j, o->shape, o->rank, cc);
          int64_t v = cc[nd->attrs[0]];
          if (is_float(o->dt)) ((float*)o->v)[j] = rnd_dt((long double)v, o->dt);
          else put_int(o, j, v);
        }
        break;
      case FGT_OP_CAST:
#pragma omp parallel for num_threads(threads) schedule(static) if (o->n >= PAR_MIN)
        for (int64_t j = 0; j < o->n; ++j) cast_one(a, j, o, j);
        break;
      case FGT_OP_COMPARE:
#pragma omp parallel for num_threads(threads) schedule(static) if (o->n >= PAR_MIN)
        for (int64_t j = 0; j < o->n; ++j) {
          int r;
          if (is_float(a->dt)) {
            float x = ((float*)a->v)[j], y = ((float*)b->v)[j];
            switch (nd->predicate) {
              case FGT_CMP_EQ: r = x == y; break;
              case FGT_CMP_NE: r = x != y; break;
              case FGT_CMP_LT: r = x < y; break;
              case FGT_CMP_LE: r = x <= y; break;
              case FGT_CMP_GT: r = x > y; break;
              default: r = x >= y;
            }
          } else {
            int64_t x = geti(a, j), y = geti(b, j);
            switch (nd->predicate) {
              case FGT_CMP_EQ: r = x == y; break;
              case FGT_CMP_NE: r = x != y; break;
              case FGT_CMP_LT: r = x < y; break;
              case FGT_CMP_LE: r = x <= y; break;
              case FGT_CMP_GT: r = x > y; break;
              default: r = x >= y;
            }
          }
          ((uint8_t*)o->v)[j] = (uint8_t)r;
        }
        break;
      case FGT_OP_SELECT:
#pragma omp parallel for num_threads(threads) schedule(static) if (o->n >= PAR_MIN)
        for (int64_t j = 0; j < o->n; ++j) {
          const Buf* s = ((uint8_t*)a->v)[j] ? b : c;
          memcpy((char*)o->v + j * vsize(o->dt), (char*)s->v + j * vsize(o->dt), vsize(o->dt));
        }
        break;
      /* index transforms (src/fugatensor/ir/tensor_rules.py:124-237; out-of-range
       * gather indices read 0 and out-of-range scatter_add indices are dropped,
       * tests/test_stage2_ops.py:190-191,230-260) */
      case FGT_OP_SLICE: {
        const int r = a->rank;
        strides(a->shape, r, as);
#pragma omp parallel for num_threads(threads) schedule(static) if (o->n >= PAR_MIN) private(cc)
        for (int64_t j = 0; j < o->n; ++j) {
          unravel(j, o->shape, r, cc);
          int64_t off = 0;
          for (int k = 0; k < r; ++k) off += (nd->attrs[k] + cc[k] * nd->attrs[r + k]) * as[k];
          memcpy((char*)o->v + j * vsize(o->dt), (char*)a->v + off * vsize(o->dt), vsize(o->dt));
        }
        break;
      }
      case FGT_OP_PAD: {
        const int r = a->rank;
        strides(a->shape, r, as);
#pragma omp parallel for num_threads(threads) schedule(static) if (o->n >= PAR_MIN) private(cc)
        for (int64_t j = 0; j < o->n; ++j) {
          unravel(j, o->shape, r, cc);
          int in = 1;
          int64_t off = 0;
          for (int k = 0; k < r && in; ++k) {
            const int64_t t = cc[k] - nd->attrs[k], step = nd->attrs[r + k] + 1;
            if (t < 0 || t % step || t / step >= a->shape[k]) in = 0;
            else off += (t / step) * as[k];
          }
          const Buf* src = in ? a : b;
          memcpy((char*)o->v + j * vsize(o->dt), (char*)src->v + (in ? off : 0) * vsize(o->dt), vsize(o->dt));
        }
        break;
      }
      case FGT_OP_CONCATENATE: {
        const int ax = (int)nd->attrs[0], r = o->rank;
        int64_t bs[FGT_MAX_RANK];
        strides(a->shape, r, as);
        strides(b->shape, r, bs);
#pragma omp parallel for num_threads(threads) schedule(static) if (o->n >= PAR_MIN) private(cc)
        for (int64_t j = 0; j < o->n; ++j) {
          unravel(j, o->shape, r, cc);
          const int first = cc[ax] < a->shape[ax];
          if (!first) cc[ax] -= a->shape[ax];
          int64_t off = 0;
          for (int k = 0; k < r; ++k) off += cc[k] * (first ? as[k] : bs[k]);
          memcpy((char*)o->v + j * vsize(o->dt), (char*)(first ? a : b)->v + off * vsize(o->dt), vsize(o->dt));
        }
        break;
      }
      case FGT_OP_GATHER: {
        const int ax = (int)nd->attrs[0], ir = b->rank, pr = a->rank;
        strides(a->shape, pr, as);
        int64_t is_[FGT_MAX_RANK];
        strides(b->shape, ir, is_);
#pragma omp parallel for num_threads(threads) schedule(static) if (o->n >= PAR_MIN) private(cc)
        for (int64_t j = 0; j < o->n; ++j) {
          unravel(j, o->shape, o->rank, cc);
          int64_t ioff = 0;
          for (int k = 0; k < ir; ++k) ioff += cc[ax + k] * is_[k];
          const int64_t idx = geti(b, ioff);
          if (idx < 0 || idx >= a->shape[ax]) {
            memset((char*)o->v + j * vsize(o->dt), 0, vsize(o->dt));
            continue;
          }
          int64_t off = idx * as[ax];
          for (int k = 0; k < ax; ++k) off += cc[k] * as[k];
          for (int k = ax + 1; k < pr; ++k) off += cc[k - 1 + ir] * as[k];
          memcpy((char*)o->v + j * vsize(o->dt), (char*)a->v + off * vsize(o->dt), vsize(o->dt));
        }
        break;
      }
      case FGT_OP_SCATTER_ADD: {
        /* base + updates in update order; LITERAL rounds every add to the
         * dtype, ACCURATE sums in long double and rounds once per element */
        const int ax = (int)nd->attrs[0], ir = b->rank, br = a->rank;
        Buf u = *c;
        strides(a->shape, br, as);
        int64_t is_[FGT_MAX_RANK];
        strides(b->shape, ir, is_);
        long double* accf = NULL;
        if (is_float(o->dt) && mode == MODE_ACCURATE) {
          accf = (long double*)malloc(sizeof(long double) * (size_t)(o->n ? o->n : 1));
          for (int64_t j = 0; j < o->n; ++j) accf[j] = ((float*)a->v)[j];
        } else {
          memcpy(o->v, a->v, (size_t)o->n * vsize(o->dt));
        }
        for (int64_t j = 0; j < u.n; ++j) {
          unravel(j, u.shape, u.rank, cc);
          int64_t ioff = 0;
          for (int k = 0; k < ir; ++k) ioff += cc[ax + k] * is_[k];
          const int64_t idx = geti(b, ioff);
          if (idx < 0 || idx >= a->shape[ax]) continue;
          int64_t off = idx * as[ax];
          for (int k = 0; k < ax; ++k) off += cc[k] * as[k];
          for (int k = ax + 1; k < br; ++k) off += cc[k - 1 + ir] * as[k];
          if (accf) accf[off] += ((float*)u.v)[j];
          else if (is_float(o->dt)) ((float*)o->v)[off] = rnd_f(((float*)o->v)[off] + ((float*)u.v)[j], o->dt);
          else put_int(o, off, wrap((int64_t)((uint64_t)geti(o, off) + (uint64_t)geti(&u, j)), o->dt));
        }
        if (accf) {
          for (int64_t j = 0; j < o->n; ++j) ((float*)o->v)[j] = rnd_dt(accf[j], o->dt);
          free(accf);
        }
        break;
      }
      default:
        if (op >= FGT_OP_REDUCE_SUM && op <= FGT_OP_ARGMIN) {
          rc = eval_reduce(nd, a, o, mode, threads);
        } else if (op >= FGT_OP_ADD && op <= FGT_OP_SHIFT_RIGHT) {
#pragma omp parallel for num_threads(threads) schedule(static) if (o->n >= PAR_MIN)
          for (int64_t j = 0; j < o->n; ++j) {
            if (is_float(o->dt)) ((float*)o->v)[j] = rnd_f(f_binary(op, ((float*)a->v)[j], ((float*)b->v)[j]), o->dt);
            else if (o->dt == FGT_BOOL) {
              int x = ((uint8_t*)a->v)[j], y = ((uint8_t*)b->v)[j], r = 0;
              if (op == FGT_OP_BITWISE_AND || op == FGT_OP_MINIMUM) r = x && y;
              else if (op == FGT_OP_BITWISE_OR || op == FGT_OP_MAXIMUM) r = x || y;
              else if (op == FGT_OP_BITWISE_XOR) r = x != y;
              ((uint8_t*)o->v)[j] = (uint8_t)r;
            } else put_int(o, j, i_binary(op, geti(a, j), geti(b, j), o->dt));
          }
        } else if (op >= FGT_OP_EXP && op <= FGT_OP_BITWISE_NOT) {
#pragma omp parallel for num_threads(threads) schedule(static) if (o->n >= PAR_MIN)
          for (int64_t j = 0; j < o->n; ++j) {
            if (is_float(o->dt)) ((float*)o->v)[j] = rnd_f(f_unary(op, ((float*)a->v)[j]), o->dt);
            else if (o->dt == FGT_BOOL) ((uint8_t*)o->v)[j] = !((uint8_t*)a->v)[j];
            else if (op == FGT_OP_ABS) {
              int64_t x = geti(a, j);
              put_int(o, j, x < 0 ? wrap((int64_t)(0 - (uint64_t)x), o->dt) : x);
            } else put_int(o, j, ~geti(a, j));
          }
        } else {
          seterr(err, errcap, "oracle: unsupported opcode");
          rc = 1;
        }
    }
    (void)xc;
    for (int k = 0; k < nd->num_operands; ++k) {
      int a_id = nd->operands[k];
      if (last[a_id] == i && B[a_id].v) {
        free(B[a_id].v);
        B[a_id].v = NULL;
      }
    }
  }
  if (!rc)
    for (int k = 0; k < d->num_outputs; ++k) store_output(&B[d->outputs[k]], outputs[k], threads);
  for (int i = 0; i < N; ++i) free(B[i].v);
  free(B);
  free(last);
  return rc;
}

int fgt_oracle_eval(const fgt_partition_desc* d, int mode, const void* const* inputs, void* const* outputs, char* err,
                    size_t errcap) {
  return eval_impl(d, mode, inputs, outputs, err, errcap, 1);
}

/* The same evaluation on `threads` OpenMP threads. */
int fgt_oracle_eval_mt(const fgt_partition_desc* d, int mode, const void* const* inputs, void* const* outputs,
                       char* err, size_t errcap, int threads) {
  return eval_impl(d, mode, inputs, outputs, err, errcap, threads);
}
