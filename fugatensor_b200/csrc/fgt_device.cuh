// fgt_device.cuh — hand-written sm_100a device library shared by every
// specialised partition kernel.
//
// The kernel generator (fgt_codegen.cpp) emits one kernel per fused kernel of
// a partition; each includes this file verbatim (NVRTC, no other headers) and
// uses only what is defined here:
//   - storage codecs for f16/bf16 (RNE through cvt.rn.*) and the reference's
//     cast rules (saturating float->int with NaN -> 0, int -> narrow float
//     rounded once, tests/backend/support/pointwise.py:239-253);
//   - IEEE maximum/minimum (NaN wins, +0 beats -0 for max; reference
//     tests/support/reduction_max.py:64-70) and first-occurrence, NaN-first
//     argmax/argmin ordering (tests/test_stage2_ops.py:148-157);
//   - 128-bit vectorised global loads/stores with an L2 evict-first hint for
//     streamed data;
//   - lane-group (xor butterfly) and block reductions.
// Floating arithmetic is IEEE with no FMA contraction: kernels are compiled
// with -fmad=false (reference: fp_contract off, src/fugatensor/_ask/gpu.py:189).
#pragma once

typedef unsigned char fgt_u8;
typedef unsigned short fgt_u16;
typedef unsigned int fgt_u32;
typedef unsigned long long fgt_u64;
typedef long long fgt_i64;

#define FGT_DEV static __device__ __forceinline__

// ---------------------------------------------------------------- codecs ---
FGT_DEV float fgt_f16_to_f32(fgt_u16 h) {
  float f;
  asm("cvt.f32.f16 %0, %1;" : "=f"(f) : "h"(h));
  return f;
}
// Narrowing uses the packed two-value conversions (cvt.rn.{f16,bf16}x2.f32)
// with +0 as the other value: on B200 they run on a faster pipe than the
// one-value forms (measured ~48 against ~16 roundings per clock per SM), and
// the rounding is the same RNE with canonical NaN. +0 converts to 0x0000.
FGT_DEV fgt_u16 fgt_f32_to_f16(float f) {
  fgt_u32 u;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(u) : "f"(0.0f), "f"(f));  // f -> low half
  return (fgt_u16)u;
}
FGT_DEV float fgt_bf16_to_f32(fgt_u16 h) { return __uint_as_float(((fgt_u32)h) << 16); }
// bf16 rounding of f as an f32 image: f goes to the high half, so the packed
// word itself is the rounded value (its low half is +0's 0x0000).
FGT_DEV float fgt_rnd_bf16(float f) {
  fgt_u32 u;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(u) : "f"(f), "f"(0.0f));
  return __uint_as_float(u);
}
FGT_DEV fgt_u16 fgt_f32_to_bf16(float f) { return (fgt_u16)(__float_as_uint(fgt_rnd_bf16(f)) >> 16); }
// Values of f16/bf16 type are carried in f32 registers, always exactly
// representable in the narrow format: every operation rounds once.
FGT_DEV float fgt_rnd_f16(float f) { return fgt_f16_to_f32(fgt_f32_to_f16(f)); }
// Storage of a value that is already an exact bf16: its high half.
FGT_DEV fgt_u16 fgt_bf16_bits_exact(float f) { return (fgt_u16)(__float_as_uint(f) >> 16); }

// Round-to-odd f32 image of an integer: narrow rounding of it afterwards is a
// single correct rounding (the narrow formats keep <= 11 significand bits).
FGT_DEV float fgt_i64_to_f32_odd(fgt_i64 x) {
  float t;
  asm("cvt.rz.f32.s64 %0, %1;" : "=f"(t) : "l"(x));
  fgt_i64 back;
  asm("cvt.rzi.s64.f32 %0, %1;" : "=l"(back) : "f"(t));
  if (back != x) t = __uint_as_float(__float_as_uint(t) | 1u);
  return t;
}
FGT_DEV float fgt_i64_to_f16v(fgt_i64 x) { return fgt_rnd_f16(fgt_i64_to_f32_odd(x)); }
FGT_DEV float fgt_i64_to_bf16v(fgt_i64 x) { return fgt_rnd_bf16(fgt_i64_to_f32_odd(x)); }
// i32 -> f16: |x| < 2^24 converts to f32 exactly (one f16 rounding follows);
// |x| >= 2^24 is beyond f16's range and rounds to +-inf either way.
FGT_DEV float fgt_i32_to_f16v(int x) { return fgt_rnd_f16((float)x); }
FGT_DEV float fgt_i32_to_bf16v(int x) {
  float t;
  asm("cvt.rz.f32.s32 %0, %1;" : "=f"(t) : "r"(x));
  int back;
  asm("cvt.rzi.s32.f32 %0, %1;" : "=r"(back) : "f"(t));
  if (back != x) t = __uint_as_float(__float_as_uint(t) | 1u);
  return fgt_rnd_bf16(t);
}

// Round-to-odd f32 image of a double (same single-rounding argument).
FGT_DEV float fgt_f64_to_f32_odd(double d) {
  float t = __double2float_rz(d);
  if ((double)t != d && t == t) t = __uint_as_float(__float_as_uint(t) | 1u);
  return t;
}

// Saturating truncation; NaN maps to 0 (the hardware's 64-bit conversion
// maps NaN to the minimum, so NaN is tested explicitly for both widths).
FGT_DEV int fgt_f32_to_i32(float f) {
  int r;
  asm("cvt.rzi.sat.s32.f32 %0, %1;" : "=r"(r) : "f"(f));
  return f != f ? 0 : r;
}
FGT_DEV fgt_i64 fgt_f32_to_i64(float f) {
  fgt_i64 r;
  asm("cvt.rzi.sat.s64.f32 %0, %1;" : "=l"(r) : "f"(f));
  return f != f ? 0 : r;
}

// ------------------------------------------------------- IEEE extrema ------
// max.NaN / min.NaN return the canonical NaN if either input is NaN and
// order -0 below +0 (checked on sm_100a for every signed-zero and NaN pair),
// which is exactly the reference's IEEE maximum/minimum.
FGT_DEV float fgt_fmax(float a, float b) {
  float r;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}
FGT_DEV float fgt_fmin(float a, float b) {
  float r;
  asm("min.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}

// Division by a value that is constant over many elements (a row statistic,
// a broadcast parameter): y = RN(1/d) is computed once with an IEEE division;
// per element q = RN(x*y), r = x - q*d (exact, by FMA), q' = RN(q + r*y).
// By Markstein's theorem (P. Markstein, "Computation of elementary functions
// on the IBM RISC System/6000 processor", IBM J. Res. Dev. 34(1), 1990) q' is
// the correctly rounded x/d when no intermediate underflows or overflows; the
// guard sends zero, tiny, huge, inf and NaN quotients (and non-normal d, for
// which y is made NaN) to the IEEE division, so the result always equals
// __fdiv_rn(x, d).
FGT_DEV float fgt_recip_for_div(float d) {
  const float a = fabsf(d);
  return (a >= 1.17549435e-38f && a <= 3.40282347e+38f) ? __fdiv_rn(1.0f, d) : __int_as_float(0x7fc00000);
}
FGT_DEV float fgt_div_by(float x, float d, float y) {
  const float q = __fmul_rn(x, y);
  const float r = __fmaf_rn(-q, d, x);
  const float q2 = __fmaf_rn(r, y, q);
  const float a = fabsf(q2);
  return (a >= 7.52316385e-37f && a <= 1.32922800e+36f) ? q2 : __fdiv_rn(x, d);
}
// The same corrected product without the guard, for phases that check the
// range once per thread (fgt_div_note / fgt_div_ok) and redo the phase with
// IEEE division (fgt_div_ieee) when a quotient left it. NaN in the max
// tracker (max.NaN) and zero or tiny quotients in the min tracker fail the
// check, so every case the guard sends to __fdiv_rn is redone.
FGT_DEV float fgt_div_q(float x, float d, float y) {
  const float q = __fmul_rn(x, y);
  const float r = __fmaf_rn(-q, d, x);
  return __fmaf_rn(r, y, q);
}
// fgt_div_q on two lanes at once (packed f32x2 multiply and FMAs; the same
// IEEE operations per lane): x - q*d is formed as fma(q, -d, x), the same
// exact value rounded once.
FGT_DEV float2 fgt_div_q2(float2 x, float d, float y) {
  const float2 yy = make_float2(y, y);
  const float2 q = __fmul2_rn(x, yy);
  const float2 r = __ffma2_rn(q, make_float2(-d, -d), x);
  return __ffma2_rn(r, yy, q);
}
// e^x for |x| <= 86 (phases note max |x| and redo with expf past it, or for
// a NaN / inf argument). x log2(e) = n + f with n the nearest integer (the
// product rounded at unit precision by adding 1.5 * 2^23) and f from the
// two-constant product x * (L2E + L2E_LO) - n (Cody & Waite's splitting, the
// error of f below 2^-24); 2^f in [2^-1/2, 2^1/2] by ex2.approx, and 2^n added
// to its exponent field: the low bits of t are n (t = 1.5 * 2^23 + n), so
// (bits(t) << 23) is n << 23 modulo 2^32 and the result stays normal.
// Error within about 2 ulp of e^x (the approximation of 2^f dominates).
FGT_DEV float fgt_ex2_approx(float f) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(f));
  return r;
}
// bits(p) + (bits(t) << 23) as one integer multiply-add (FMA pipe) rather
// than a shift and an add (ALU pipe); the same bits modulo 2^32
FGT_DEV float fgt_exp_scale(float p, float t) {
  int r;
  asm("mad.lo.s32 %0, %1, 8388608, %2;" : "=r"(r) : "r"(__float_as_int(t)), "r"(__float_as_int(p)));
  return __int_as_float(r);
}
FGT_DEV float fgt_exp_q(float x) {
  const float t = __fmaf_rn(x, __int_as_float(0x3fb8aa3b), __int_as_float(0x4b400000));
  const float nn = __fsub_rn(__int_as_float(0x4b400000), t);  // -n, exact
  const float f = __fmaf_rn(x, __int_as_float(0x32a57060), __fmaf_rn(x, __int_as_float(0x3fb8aa3b), nn));
  return fgt_exp_scale(fgt_ex2_approx(f), t);
}
FGT_DEV float2 fgt_exp_q2(float2 x) {
  const float2 t = __ffma2_rn(x, make_float2(__int_as_float(0x3fb8aa3b), __int_as_float(0x3fb8aa3b)), make_float2(__int_as_float(0x4b400000), __int_as_float(0x4b400000)));
  const float2 nn = __ffma2_rn(t, make_float2(-1.0f, -1.0f), make_float2(__int_as_float(0x4b400000), __int_as_float(0x4b400000)));
  const float2 f1 = __ffma2_rn(x, make_float2(__int_as_float(0x3fb8aa3b), __int_as_float(0x3fb8aa3b)), nn);
  const float2 f = __ffma2_rn(x, make_float2(__int_as_float(0x32a57060), __int_as_float(0x32a57060)), f1);
  return make_float2(fgt_exp_scale(fgt_ex2_approx(f.x), t.x), fgt_exp_scale(fgt_ex2_approx(f.y), t.y));
}
// Warp-wide f32 max / min in one instruction (sm_100a redux.sync with .NaN:
// a NaN input gives NaN), the same IEEE maximum / minimum as fgt_fmax /
// fgt_fmin over the warp's 32 values.
FGT_DEV float fgt_redux_max(float x) {
  float r;
  asm("redux.sync.max.NaN.f32 %0, %1, 0xffffffff;" : "=f"(r) : "f"(x));
  return r;
}
FGT_DEV float fgt_redux_min(float x) {
  float r;
  asm("redux.sync.min.NaN.f32 %0, %1, 0xffffffff;" : "=f"(r) : "f"(x));
  return r;
}
FGT_DEV void fgt_exp_note(float& mx, float x) { mx = fgt_fmax(mx, fabsf(x)); }
FGT_DEV bool fgt_exp_ok(float mx) { return mx <= 86.0f; }
FGT_DEV void fgt_div_note(float& mx, float& mn, float q) {
  mx = fgt_fmax(mx, fabsf(q));
  mn = fminf(mn, fabsf(q));
}
// Both lanes of a pair noted at once: sm_100's three-input max.NaN / min
// (PTX ISA 8.8), the same values as two fgt_div_note / fgt_exp_note steps.
FGT_DEV void fgt_div_note2(float& mx, float& mn, float a, float b) {
  asm("max.NaN.f32 %0, %1, %2, %3;" : "=f"(mx) : "f"(mx), "f"(fabsf(a)), "f"(fabsf(b)));
  asm("min.f32 %0, %1, %2, %3;" : "=f"(mn) : "f"(mn), "f"(fabsf(a)), "f"(fabsf(b)));
}
FGT_DEV void fgt_exp_note2(float& mx, float a, float b) {
  asm("max.NaN.f32 %0, %1, %2, %3;" : "=f"(mx) : "f"(mx), "f"(fabsf(a)), "f"(fabsf(b)));
}
// Narrow division (x * RN(1/d), partitions with only 16-bit floating
// outputs): usable while the row's reciprocal is a number (fgt_recip_for_div
// returns NaN for a divisor without a normal reciprocal).
FGT_DEV bool fgt_rcp_ok(float y) { return y == y; }
FGT_DEV float fgt_div_nby(float x, float d, float y) { return y == y ? __fmul_rn(x, y) : __fdiv_rn(x, d); }
FGT_DEV bool fgt_div_ok(float mx, float mn) { return mx <= 1.32922800e+36f && mn >= 7.52316385e-37f; }
FGT_DEV float fgt_div_ieee(float x, float d, float) { return __fdiv_rn(x, d); }
// Max / min of a packed accumulator with a register row piece of N bf16
// values, two values per instruction (max.NaN / min.NaN on bf16x2: NaN wins,
// exact otherwise). The halves are folded into the f32 accumulator later.
// 16-bit element v of a packed row piece (two values per 32-bit word, the
// lower index in the low half)
template <int N> FGT_DEV fgt_u16 fgt_h16(const fgt_u32 (&w)[N], int v) { return (fgt_u16)(w[v >> 1] >> ((v & 1) * 16)); }
// ---- programmatic dependent launch ----------------------------------------
// Every kernel starts here. The next kernel on the stream, when it is launched
// with programmatic stream serialization, may be scheduled once every CTA of
// this grid has started (its CTAs wait in whatever room this grid leaves on
// the SMs), and this grid waits until the grid before it has completed with its memory
// visible before it reads anything. Without that launch attribute both
// instructions do nothing.
FGT_DEV void fgt_pdl_enter() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
// ---- peer mailboxes (records exchanged between ranks over NVLink) --------
FGT_DEV unsigned long long fgt_globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;\n" : "=l"(t));
  return t;
}
// A failed exchange: the host-mapped status word of the communicator.
FGT_DEV void fgt_xfail(unsigned* status) {
  *(volatile unsigned*)status = 1u;
  __threadfence_system();
}

// ---- record words of the peer exchange -------------------------------------
// A rank's record travels as 8-byte words, each holding 4 bytes of data in its
// low half and the launch's epoch in its high half, written and read with
// single 64-bit accesses (naturally aligned 64-bit scalar accesses are
// single-copy atomic). A reader that sees the epoch in a word therefore sees
// that word's data: no fence and no separate flag are needed, as in NCCL's
// low-latency protocol. Every record value owns 8 record bytes at an 8-byte
// offset b, carried by the two words at bytes 2b and 2b + 8 of the slot
// (narrower values use the first word only, zero-extended).
FGT_DEV void fgt_ll_store(unsigned char* slot, fgt_i64 byte_off, fgt_u32 v, unsigned ep) {
  const fgt_u64 w = ((fgt_u64)ep << 32) | v;
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;\n" ::"l"(slot + 2 * byte_off), "l"(w) : "memory");
}
// Waits, until t0 + limit ns, for the word to carry epoch `ep`; on timeout the
// status word is set and whatever the word holds is returned.
FGT_DEV fgt_u32 fgt_ll_load(const unsigned char* slot, fgt_i64 byte_off, unsigned ep, unsigned long long t0,
                            unsigned long long limit, unsigned* status) {
  fgt_u64 w;
  for (;;) {
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];\n" : "=l"(w) : "l"(slot + 2 * byte_off) : "memory");
    if ((unsigned)(w >> 32) == ep) break;
    if (fgt_globaltimer() - t0 > limit) {
      fgt_xfail(status);
      break;
    }
    __nanosleep(32);
  }
  return (fgt_u32)w;
}
// A word read without waiting (all of a record's words are requested before
// any is checked, so their latencies overlap), and its value once it carries
// `ep`: taken as read, or waited for as fgt_ll_load does.
FGT_DEV fgt_u64 fgt_ll_raw(const unsigned char* slot, fgt_i64 byte_off) {
  fgt_u64 w;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];\n" : "=l"(w) : "l"(slot + 2 * byte_off) : "memory");
  return w;
}
FGT_DEV fgt_u32 fgt_ll_take(fgt_u64 w, const unsigned char* slot, fgt_i64 byte_off, unsigned ep, unsigned long long t0,
                            unsigned long long limit, unsigned* status) {
  if ((unsigned)(w >> 32) == ep) return (fgt_u32)w;
  return fgt_ll_load(slot, byte_off, ep, t0, limit, status);
}
// Bit images of the record value types (8 bytes wide, narrower ones zero-extended).
FGT_DEV fgt_u64 fgt_bits64(float v) { return __float_as_uint(v); }
FGT_DEV fgt_u64 fgt_bits64(double v) { return (fgt_u64)__double_as_longlong(v); }
FGT_DEV fgt_u64 fgt_bits64(fgt_i64 v) { return (fgt_u64)v; }
FGT_DEV fgt_u64 fgt_bits64(fgt_u64 v) { return v; }
FGT_DEV fgt_u64 fgt_bits64(int v) { return (fgt_u32)v; }
FGT_DEV fgt_u64 fgt_bits64(fgt_u32 v) { return v; }
FGT_DEV fgt_u64 fgt_bits64(fgt_u16 v) { return v; }
FGT_DEV fgt_u64 fgt_bits64(fgt_u8 v) { return v; }
FGT_DEV fgt_u64 fgt_bits64(bool v) { return v ? 1u : 0u; }
template <typename T> FGT_DEV void fgt_from_bits64(fgt_u64 b, T& out) { out = (T)b; }
FGT_DEV void fgt_from_bits64(fgt_u64 b, float& out) { out = __uint_as_float((fgt_u32)b); }
FGT_DEV void fgt_from_bits64(fgt_u64 b, double& out) { out = __longlong_as_double((long long)b); }
template <typename T> FGT_DEV void fgt_ll_put(unsigned char* slot, fgt_i64 byte_off, T v, unsigned ep) {
  const fgt_u64 b = fgt_bits64(v);
  fgt_ll_store(slot, byte_off, (fgt_u32)b, ep);
  if (sizeof(T) == 8) fgt_ll_store(slot, byte_off + 4, (fgt_u32)(b >> 32), ep);
}
template <typename T>
FGT_DEV T fgt_ll_value(fgt_u64 w0, fgt_u64 w1, const unsigned char* slot, fgt_i64 byte_off, unsigned ep, unsigned long long t0,
                       unsigned long long limit, unsigned* status) {
  fgt_u64 b = fgt_ll_take(w0, slot, byte_off, ep, t0, limit, status);
  if (sizeof(T) == 8) b |= (fgt_u64)fgt_ll_take(w1, slot, byte_off + 4, ep, t0, limit, status) << 32;
  T r;
  fgt_from_bits64(b, r);
  return r;
}
template <typename T>
FGT_DEV T fgt_ll_get(const unsigned char* slot, fgt_i64 byte_off, unsigned ep, unsigned long long t0, unsigned long long limit,
                     unsigned* status) {
  fgt_u64 b = fgt_ll_load(slot, byte_off, ep, t0, limit, status);
  if (sizeof(T) == 8) b |= (fgt_u64)fgt_ll_load(slot, byte_off + 4, ep, t0, limit, status) << 32;
  T r;
  fgt_from_bits64(b, r);
  return r;
}

// Element v of a packed 16-bit array (v a compile-time constant after unrolling).
// A copy of a register value that the compiler cannot see through (an empty
// volatile asm that claims to modify it): values a later row phase derives
// from it are not recognised as equal to the earlier phases', so each phase
// recomputes them instead of the compiler keeping them live across the row's
// barriers. No instruction is emitted.
FGT_DEV void fgt_opaque(float& x) { asm volatile("" : "+f"(x)); }
FGT_DEV void fgt_opaque(double& x) { asm volatile("" : "+d"(x)); }
FGT_DEV void fgt_opaque(fgt_u32& x) { asm volatile("" : "+r"(x)); }
FGT_DEV void fgt_opaque(int& x) { asm volatile("" : "+r"(x)); }
FGT_DEV void fgt_opaque(fgt_i64& x) { asm volatile("" : "+l"(x)); }
FGT_DEV void fgt_opaque(fgt_u64& x) { asm volatile("" : "+l"(x)); }
FGT_DEV void fgt_opaque(fgt_u16& x) { asm volatile("" : "+h"(x)); }
FGT_DEV void fgt_opaque(fgt_u8&) {}
template <int N> FGT_DEV void fgt_set_h16(fgt_u32 (&w)[N], int v, fgt_u16 h) {
  w[v >> 1] = (v & 1) ? ((w[v >> 1] & 0xffffu) | ((fgt_u32)h << 16)) : ((w[v >> 1] & 0xffff0000u) | (fgt_u32)h);
}
// packed pieces are already bf16x2 words
template <int N> FGT_DEV fgt_u32 fgt_max_bf16x2_row(fgt_u32 acc, const fgt_u32 (&w)[N]) {
#pragma unroll
  for (int k = 0; k < N; ++k) asm("max.NaN.bf16x2 %0, %1, %2;" : "=r"(acc) : "r"(acc), "r"(w[k]));
  return acc;
}
template <int N> FGT_DEV fgt_u32 fgt_min_bf16x2_row(fgt_u32 acc, const fgt_u32 (&w)[N]) {
#pragma unroll
  for (int k = 0; k < N; ++k) asm("min.NaN.bf16x2 %0, %1, %2;" : "=r"(acc) : "r"(acc), "r"(w[k]));
  return acc;
}
template <int N> FGT_DEV fgt_u32 fgt_max_bf16x2_row(fgt_u32 acc, const fgt_u16 (&h)[N]) {
  static_assert(N % 2 == 0, "pairs");
#pragma unroll
  for (int k = 0; k < N; k += 2) {
    const fgt_u32 w = (fgt_u32)h[k] | ((fgt_u32)h[k + 1] << 16);
    asm("max.NaN.bf16x2 %0, %1, %2;" : "=r"(acc) : "r"(acc), "r"(w));
  }
  return acc;
}
template <int N> FGT_DEV fgt_u32 fgt_min_bf16x2_row(fgt_u32 acc, const fgt_u16 (&h)[N]) {
  static_assert(N % 2 == 0, "pairs");
#pragma unroll
  for (int k = 0; k < N; k += 2) {
    const fgt_u32 w = (fgt_u32)h[k] | ((fgt_u32)h[k + 1] << 16);
    asm("min.NaN.bf16x2 %0, %1, %2;" : "=r"(acc) : "r"(acc), "r"(w));
  }
  return acc;
}
// ---- thread-block clusters: a row split over the CTAs of a cluster combines
// its reductions through distributed shared memory (DSMEM).
FGT_DEV unsigned fgt_cluster_rank() {
  unsigned r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// All threads of every CTA of the cluster: writes before it are visible to
// DSMEM reads after it.
FGT_DEV void fgt_cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;\n" ::: "memory");
}
// Value of `local`'s shared-memory location in CTA `rank` of the cluster.
template <class T> FGT_DEV T fgt_dsmem_ld(const T* local, unsigned rank) {
  static_assert(sizeof(T) == 4 || sizeof(T) == 8, "32- or 64-bit values");
  const unsigned la = (unsigned)__cvta_generic_to_shared(local);
  unsigned ra;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(la), "r"(rank));
  union { T v; unsigned u[sizeof(T) / 4]; } w;
  if (sizeof(T) == 4) {
    asm volatile("ld.shared::cluster.b32 %0, [%1];" : "=r"(w.u[0]) : "r"(ra) : "memory");
  } else {
    unsigned long long b;
    asm volatile("ld.shared::cluster.b64 %0, [%1];" : "=l"(b) : "r"(ra) : "memory");
    w.u[0] = (unsigned)b;
    w.u[sizeof(T) / 4 - 1] = (unsigned)(b >> 32);
  }
  return w.v;
}
template <class T> FGT_DEV T fgt_imax(T a, T b) { return a > b ? a : b; }
template <class T> FGT_DEV T fgt_imin(T a, T b) { return a < b ? a : b; }

// Is (a, ia) strictly preferred over (b, ib) for argmax (MAX=true) / argmin?
// NaN counts as the extremum; ties keep the lowest index.
template <bool MAX, class I> FGT_DEV bool fgt_arg_better_f(float a, I ia, float b, I ib) {
  const bool an = a != a, bn = b != b;
  if (an || bn) return (an && bn) ? ia < ib : an;
  if (MAX ? a > b : a < b) return true;
  if (MAX ? a < b : a > b) return false;
  return ia < ib;
}
template <bool MAX, class T, class I> FGT_DEV bool fgt_arg_better_i(T a, I ia, T b, I ib) {
  if (MAX ? a > b : a < b) return true;
  if (MAX ? a < b : a > b) return false;
  return ia < ib;
}

// --------------------------------------------------- integer semantics ----
// Wrapping arithmetic and the reference's floordiv/mod/shift definitions
// (tests/support/stage2.py:36-67): division by zero gives 0; MIN // -1 = MIN.
template <class T, class U> FGT_DEV T fgt_wrap_add(T a, T b) { return (T)((U)a + (U)b); }
template <class T, class U> FGT_DEV T fgt_wrap_mul(T a, T b) { return (T)((U)a * (U)b); }
template <class T> FGT_DEV T fgt_ifloordiv(T a, T b, T minv) {
  if (b == 0) return 0;
  if (a == minv && b == (T)-1) return minv;
  T q = a / b;
  if ((a % b != 0) && ((a < 0) != (b < 0))) q -= 1;
  return q;
}
template <class T> FGT_DEV T fgt_imod(T a, T b, T minv) {
  if (b == 0) return 0;
  if (a == minv && b == (T)-1) return 0;
  T r = a % b;
  if (r != 0 && ((r < 0) != (b < 0))) r += b;
  return r;
}
template <class T, class U, int BITS> FGT_DEV T fgt_ishl(T a, T b) {
  if (b < 0 || b >= BITS) return 0;
  return (T)((U)a << b);
}
template <class T, int BITS> FGT_DEV T fgt_ishr(T a, T b) {
  if (b < 0) return 0;
  if (b >= BITS) return a < 0 ? (T)-1 : (T)0;
  return a >> b;
}
template <class T, class U> FGT_DEV T fgt_ipow(T base, T e) {
  if (e < 0) {
    if (base == 1) return 1;
    if (base == (T)-1) return (e & 1) ? (T)-1 : (T)1;
    return 0;
  }
  U result = 1, b = (U)base;
  while (e) {
    if (e & 1) result *= b;
    b *= b;
    e >>= 1;
  }
  return (T)result;
}
FGT_DEV float fgt_ffloordiv(float a, float b) { return floorf(__fdiv_rn(a, b)); }
FGT_DEV float fgt_fmod_py(float a, float b) {
  float r = fmodf(a, b);
  if (r != 0.0f && ((r < 0.0f) != (b < 0.0f))) r = __fadd_rn(r, b);
  return r;
}

// ------------------------------------------------------ vector memory -----
// 16-byte vector accesses. Streamed inputs are read once: evict-first keeps
// them from displacing reused data (broadcast operands, partials) in L2.
template <int BYTES> struct fgt_vec_t;
template <> struct fgt_vec_t<16> { typedef uint4 type; };
template <> struct fgt_vec_t<8> { typedef uint2 type; };
template <> struct fgt_vec_t<4> { typedef unsigned int type; };
template <> struct fgt_vec_t<2> { typedef unsigned short type; };
template <> struct fgt_vec_t<1> { typedef unsigned char type; };

template <class T, int N> FGT_DEV void fgt_vload(T (&dst)[N], const T* __restrict__ src) {
  typedef typename fgt_vec_t<sizeof(T) * N>::type V;
  union { V v; T e[N]; } u;
  u.v = __ldcs(reinterpret_cast<const V*>(src));
#pragma unroll
  for (int k = 0; k < N; ++k) dst[k] = u.e[k];
}
template <class T, int N> FGT_DEV void fgt_vload_keep(T (&dst)[N], const T* __restrict__ src) {
  typedef typename fgt_vec_t<sizeof(T) * N>::type V;
  union { V v; T e[N]; } u;
  u.v = __ldg(reinterpret_cast<const V*>(src));
#pragma unroll
  for (int k = 0; k < N; ++k) dst[k] = u.e[k];
}
template <class T, int N> FGT_DEV void fgt_vstore(T* __restrict__ dst, const T (&src)[N]) {
  typedef typename fgt_vec_t<sizeof(T) * N>::type V;
  union { V v; T e[N]; } u;
#pragma unroll
  for (int k = 0; k < N; ++k) u.e[k] = src[k];
  __stcs(reinterpret_cast<V*>(dst), u.v);
}
// Store N f32 values rounded to bf16: each pair is rounded and packed by one
// cvt.rn.bf16x2.f32 (the same RNE as the one-value rounding).
template <int N> FGT_DEV void fgt_vstore_bf16_rn(fgt_u16* __restrict__ dst, const float (&src)[N]) {
  static_assert(N % 2 == 0, "pairs");
  typedef typename fgt_vec_t<2 * N>::type V;
  union { V v; fgt_u32 w[N / 2]; } u;
#pragma unroll
  for (int k = 0; k < N / 2; ++k) asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(u.w[k]) : "f"(src[2 * k + 1]), "f"(src[2 * k]));
  __stcs(reinterpret_cast<V*>(dst), u.v);
}

// --------------------------------------------- shared-memory row staging ---
// Streamed row operands are copied global -> shared with cp.async in a ring of
// stages, several rows ahead of the row being computed. Every thread copies
// and later reads back only its own pieces, so completion is tracked per
// thread (cp.async.wait_group) and no block barrier is involved; data in
// flight occupies shared memory, not registers.
FGT_DEV unsigned fgt_smem_addr(const void* p) { return (unsigned)__cvta_generic_to_shared(p); }
// ---- tensor memory (TMEM) as per-thread storage --------------------------
// A CTA allocates columns of the SM's tensor memory (128 lanes x 512 columns
// of 32 bits) with one warp; a warp of a 32x32b access reaches only the 32
// lanes of its quarter (warp id mod 4), and each thread its own lane. Row
// kernels keep column-reduction accumulators there: thread t of warp w owns
// lane 32 * (w % 4) + t and a private column range chosen by w / 4, and moves
// one chunk of accumulators to registers and back per update. tcgen05.ld is
// asynchronous: the load and its wait are one asm statement, so no use of
// the registers can be scheduled before the data has arrived.
FGT_DEV void fgt_tm_alloc(unsigned* slot, unsigned ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(fgt_smem_addr(slot)), "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
}
FGT_DEV void fgt_tm_dealloc(unsigned base, unsigned ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(base), "r"(ncols) : "memory");
}
FGT_DEV void fgt_tm_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory"); }
FGT_DEV void fgt_tm_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory"); }
FGT_DEV void fgt_tm_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory"); }
FGT_DEV void fgt_tm_ld(float (&r)[4], unsigned a) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];\ntcgen05.wait::ld.sync.aligned;\n"
               : "=f"(r[0]), "=f"(r[1]), "=f"(r[2]), "=f"(r[3])
               : "r"(a)
               : "memory");
}
FGT_DEV void fgt_tm_st(unsigned a, const float (&r)[4]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1,%2,%3,%4};\n" ::"r"(a), "f"(r[0]), "f"(r[1]), "f"(r[2]), "f"(r[3])
               : "memory");
}
FGT_DEV void fgt_tm_ld(float (&r)[8], unsigned a) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];\ntcgen05.wait::ld.sync.aligned;\n"
               : "=f"(r[0]), "=f"(r[1]), "=f"(r[2]), "=f"(r[3]), "=f"(r[4]), "=f"(r[5]), "=f"(r[6]), "=f"(r[7])
               : "r"(a)
               : "memory");
}
FGT_DEV void fgt_tm_st(unsigned a, const float (&r)[8]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};\n" ::"r"(a), "f"(r[0]), "f"(r[1]),
               "f"(r[2]), "f"(r[3]), "f"(r[4]), "f"(r[5]), "f"(r[6]), "f"(r[7])
               : "memory");
}
FGT_DEV void fgt_tm_ld(float (&r)[16], unsigned a) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
      "tcgen05.wait::ld.sync.aligned;\n"
      : "=f"(r[0]), "=f"(r[1]), "=f"(r[2]), "=f"(r[3]), "=f"(r[4]), "=f"(r[5]), "=f"(r[6]), "=f"(r[7]), "=f"(r[8]), "=f"(r[9]),
        "=f"(r[10]), "=f"(r[11]), "=f"(r[12]), "=f"(r[13]), "=f"(r[14]), "=f"(r[15])
      : "r"(a)
      : "memory");
}
FGT_DEV void fgt_tm_st(unsigned a, const float (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};\n" ::"r"(a),
      "f"(r[0]), "f"(r[1]), "f"(r[2]), "f"(r[3]), "f"(r[4]), "f"(r[5]), "f"(r[6]), "f"(r[7]), "f"(r[8]), "f"(r[9]), "f"(r[10]),
      "f"(r[11]), "f"(r[12]), "f"(r[13]), "f"(r[14]), "f"(r[15])
      : "memory");
}
template <int BYTES> FGT_DEV void fgt_cp_async(unsigned dst, const void* src) {
  if (BYTES == 16) asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(dst), "l"(src) : "memory");
  else asm volatile("cp.async.ca.shared.global [%0], [%1], %2;\n" ::"r"(dst), "l"(src), "n"(BYTES) : "memory");
}
FGT_DEV void fgt_cp_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N> FGT_DEV void fgt_cp_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory"); }
template <class T, int N> FGT_DEV void fgt_lds(T (&dst)[N], const T* src) {
  typedef typename fgt_vec_t<sizeof(T) * N>::type V;
  union { V v; T e[N]; } u;
  u.v = *reinterpret_cast<const V*>(src);
#pragma unroll
  for (int k = 0; k < N; ++k) dst[k] = u.e[k];
}

// Ascending-order scans (a thread visits its elements in increasing index):
// a later element replaces the running extremum only if strictly better, or
// if it is the first NaN. Equivalent to fgt_arg_better_* for such scans.
// `unset` is the sentinel index of an accumulator that holds no element yet.
template <bool MAX, class I> FGT_DEV bool fgt_arg_scan_f(float v, float best, I bi, I unset) {
  return bi == unset || (MAX ? v > best : v < best) || (v != v && best == best);
}
template <bool MAX, class T, class I> FGT_DEV bool fgt_arg_scan_i(T v, T best, I bi, I unset) {
  return bi == unset || (MAX ? v > best : v < best);
}

// ------------------------------------------------------- shuffles ---------
FGT_DEV float fgt_shfl_xor(float v, int m) { return __shfl_xor_sync(0xffffffffu, v, m); }
FGT_DEV double fgt_shfl_xor(double v, int m) { return __shfl_xor_sync(0xffffffffu, v, m); }
FGT_DEV int fgt_shfl_xor(int v, int m) { return __shfl_xor_sync(0xffffffffu, v, m); }
FGT_DEV fgt_i64 fgt_shfl_xor(fgt_i64 v, int m) { return __shfl_xor_sync(0xffffffffu, v, m); }
FGT_DEV bool fgt_shfl_xor(bool v, int m) { return __shfl_xor_sync(0xffffffffu, (int)v, m) != 0; }
