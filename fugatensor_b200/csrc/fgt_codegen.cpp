// fgt_codegen.cpp — specialising the kernel templates for one partition.
//
// Each kernel family (ELEM / ROW / COLFIN / FULLFIN, see fgt_plan.h) is a
// fixed loop skeleton written here; per partition only the element functor
// (straight-line code for one element), the index arithmetic and the
// reduction set are generated. Values are placed in the outermost scope
// where they are computable: kernel constants once per CTA, row statistics
// once per row, column operands (gamma, beta) once per CTA in registers,
// element values per lane. Streamed operands are loaded with 128-bit vector
// loads once per row and stay in registers across the row's phases.
//
// Arithmetic follows the reference's owned kernels: IEEE f32 with no FMA
// contraction (src/fugatensor/_ask/gpu.py:189), f16/bf16 computed in f32 and
// rounded once per operation, exp/log/tanh/erf through CUDA's f32 math
// library (the reference links libdevice, src/fugatensor/_ask/cuda.py:215-229).
#include <cstdio>
#include <cstring>
#include <functional>
#include <sstream>

#include "fgt_plan.h"

namespace fgt {

namespace {

std::string st_t(int dt) {
  switch (dt) {
    case FGT_BOOL: return "fgt_u8";
    case FGT_I32: return "int";
    case FGT_I64: return "fgt_i64";
    case FGT_F32: return "float";
    default: return "fgt_u16";
  }
}
std::string vt_t(int dt) {
  switch (dt) {
    case FGT_BOOL: return "bool";
    case FGT_I32: return "int";
    case FGT_I64: return "fgt_i64";
    default: return "float";
  }
}
std::string ut_t(int dt) { return dt == FGT_I64 ? "fgt_u64" : "fgt_u32"; }
std::string min_lit(int dt) { return dt == FGT_I64 ? "(-9223372036854775807LL-1LL)" : "(-2147483647-1)"; }
std::string max_lit(int dt) { return dt == FGT_I64 ? "9223372036854775807LL" : "2147483647"; }
int bits_of(int dt) { return dt == FGT_I64 ? 64 : 32; }

std::string ld_conv(int dt, const std::string& x) {
  switch (dt) {
    case FGT_F16: return "fgt_f16_to_f32(" + x + ")";
    case FGT_BF16: return "fgt_bf16_to_f32(" + x + ")";
    case FGT_BOOL: return "((" + x + ")!=0)";
    default: return x;
  }
}
// Every value of a narrow dtype is exactly representable (each operation
// rounds), so a bf16 store is the high half of its f32 image.
std::string st_conv(int dt, const std::string& x) {
  switch (dt) {
    case FGT_F16: return "fgt_f32_to_f16(" + x + ")";
    case FGT_BF16: return "fgt_bf16_bits_exact(" + x + ")";
    case FGT_BOOL: return "(fgt_u8)(" + x + ")";
    default: return x;
  }
}
std::string rnd(int dt, const std::string& x) {
  if (dt == FGT_F16) return "fgt_rnd_f16(" + x + ")";
  if (dt == FGT_BF16) return "fgt_rnd_bf16(" + x + ")";
  return x;
}

float half_bits_to_float(uint16_t h) {
  uint32_t s = (h >> 15) & 1, e = (h >> 10) & 0x1f, f = h & 0x3ff;
  uint32_t out;
  if (e == 0x1f) out = (s << 31) | 0x7f800000u | (f ? 0x400000u : 0);
  else if (e == 0) {
    if (!f) out = s << 31;
    else {
      int ex = -14;
      while (!(f & 0x400)) {
        f <<= 1;
        --ex;
      }
      f &= 0x3ff;
      out = (s << 31) | ((uint32_t)(ex + 127) << 23) | (f << 13);
    }
  } else out = (s << 31) | ((e - 15 + 127) << 23) | (f << 13);
  float r;
  std::memcpy(&r, &out, 4);
  return r;
}

std::string hex32(uint32_t v) {
  char b[32];
  std::snprintf(b, sizeof b, "0x%08xu", v);
  return b;
}

std::string literal(int dt, uint64_t bits) {
  switch (dt) {
    case FGT_BOOL: return (bits & 0xff) ? "true" : "false";
    case FGT_I32: return "((int)" + hex32((uint32_t)bits) + ")";
    case FGT_I64: {
      char b[48];
      std::snprintf(b, sizeof b, "((fgt_i64)0x%016llxULL)", (unsigned long long)bits);
      return b;
    }
    case FGT_F32: return "__uint_as_float(" + hex32((uint32_t)bits) + ")";
    case FGT_F16: {
      float f = half_bits_to_float((uint16_t)bits);
      uint32_t u;
      std::memcpy(&u, &f, 4);
      return "__uint_as_float(" + hex32(u) + ")";
    }
    case FGT_BF16: return "__uint_as_float(" + hex32(((uint32_t)(bits & 0xffff)) << 16) + ")";
  }
  return "0";
}

std::string cast_expr(int from, int to, const std::string& a) {
  if (from == to) return a;
  if (to == FGT_BOOL) return "((" + a + ")!=0)";
  if (from == FGT_BOOL) {
    if (is_float(to)) return "((" + a + ")?1.0f:0.0f)";
    return "((" + vt_t(to) + ")((" + a + ")?1:0))";
  }
  if (is_int(from) && is_int(to)) return "((" + vt_t(to) + ")(" + a + "))";
  if (is_int(from)) {
    if (to == FGT_F32) return "((float)(" + a + "))";
    // From i32: f16 overflows below 2^24, where the f32 image is still exact,
    // so one f32 conversion and one f16 rounding suffice; bf16 needs the
    // round-to-odd image, taken in 32 bits.
    if (from == FGT_I32) return to == FGT_F16 ? "fgt_i32_to_f16v(" + a + ")" : "fgt_i32_to_bf16v(" + a + ")";
    if (to == FGT_F16) return "fgt_i64_to_f16v((fgt_i64)(" + a + "))";
    return "fgt_i64_to_bf16v((fgt_i64)(" + a + "))";
  }
  // from floating
  if (to == FGT_I32) return "fgt_f32_to_i32(" + a + ")";
  if (to == FGT_I64) return "fgt_f32_to_i64(" + a + ")";
  return rnd(to, a);  // f32/f16/bf16 -> narrower or equal: one rounding
}

const char* cmp_op(int p) {
  switch (p) {
    case FGT_CMP_EQ: return "==";
    case FGT_CMP_NE: return "!=";
    case FGT_CMP_LT: return "<";
    case FGT_CMP_LE: return "<=";
    case FGT_CMP_GT: return ">";
    default: return ">=";
  }
}

std::string binary_expr(int op, int dt, const std::string& a, const std::string& b) {
  const std::string T = vt_t(dt), U = ut_t(dt);
  const bool f = is_float(dt);
  switch (op) {
    case FGT_OP_ADD: return f ? rnd(dt, "__fadd_rn(" + a + "," + b + ")") : "fgt_wrap_add<" + T + "," + U + ">(" + a + "," + b + ")";
    case FGT_OP_MUL: {
      if (!f) return "fgt_wrap_mul<" + T + "," + U + ">(" + a + "," + b + ")";
      // x * (+-1) of a value exact in its dtype is exact (it is how the
      // reference spells negation and subtraction), so it needs no rounding.
      // As a negation it folds into the consumer (an add of -x is a subtract):
      // the same value for every non-NaN x (a NaN keeps its payload, sign aside).
      static const std::string one = "__uint_as_float(0x3f800000u)", neg = "__uint_as_float(0xbf800000u)";
      if (b == one) return a;
      if (a == one) return b;
      if (b == neg) return "(-" + a + ")";
      if (a == neg) return "(-" + b + ")";
      return rnd(dt, "__fmul_rn(" + a + "," + b + ")");
    }
    case FGT_OP_DIV: {
      // x / 2^k is x * 2^-k exactly (both are one rounding of the same real)
      unsigned bits = 0;
      if (std::sscanf(b.c_str(), "__uint_as_float(0x%8xu)", &bits) == 1 && (bits & 0x7fffffu) == 0) {
        const unsigned e = (bits >> 23) & 0xffu;
        if (e >= 1 && e <= 253) {
          const unsigned r = (bits & 0x80000000u) | ((254u - e) << 23);
          char lit[48];
          std::snprintf(lit, sizeof lit, "__uint_as_float(0x%08xu)", r);
          return rnd(dt, "__fmul_rn(" + a + "," + lit + ")");
        }
      }
      return rnd(dt, "__fdiv_rn(" + a + "," + b + ")");
    }
    case FGT_OP_MAXIMUM:
      if (f) return "fgt_fmax(" + a + "," + b + ")";
      if (dt == FGT_BOOL) return "(" + a + "||" + b + ")";
      return "fgt_imax<" + T + ">(" + a + "," + b + ")";
    case FGT_OP_MINIMUM:
      if (f) return "fgt_fmin(" + a + "," + b + ")";
      if (dt == FGT_BOOL) return "(" + a + "&&" + b + ")";
      return "fgt_imin<" + T + ">(" + a + "," + b + ")";
    case FGT_OP_POW: return f ? rnd(dt, "powf(" + a + "," + b + ")") : "fgt_ipow<" + T + "," + U + ">(" + a + "," + b + ")";
    case FGT_OP_FLOORDIV:
      return f ? rnd(dt, "fgt_ffloordiv(" + a + "," + b + ")") : "fgt_ifloordiv<" + T + ">(" + a + "," + b + "," + min_lit(dt) + ")";
    case FGT_OP_MOD: return f ? rnd(dt, "fgt_fmod_py(" + a + "," + b + ")") : "fgt_imod<" + T + ">(" + a + "," + b + "," + min_lit(dt) + ")";
    case FGT_OP_BITWISE_AND: return dt == FGT_BOOL ? "(" + a + "&&" + b + ")" : "(" + a + "&" + b + ")";
    case FGT_OP_BITWISE_OR: return dt == FGT_BOOL ? "(" + a + "||" + b + ")" : "(" + a + "|" + b + ")";
    case FGT_OP_BITWISE_XOR: return dt == FGT_BOOL ? "(" + a + "!=" + b + ")" : "(" + a + "^" + b + ")";
    case FGT_OP_SHIFT_LEFT: return "fgt_ishl<" + T + "," + U + "," + std::to_string(bits_of(dt)) + ">(" + a + "," + b + ")";
    case FGT_OP_SHIFT_RIGHT: return "fgt_ishr<" + T + "," + std::to_string(bits_of(dt)) + ">(" + a + "," + b + ")";
  }
  fail(FGT_ERR_UNSUPPORTED, "binary opcode not supported by the generator");
}

std::string unary_expr(int op, int dt, const std::string& a) {
  switch (op) {
    case FGT_OP_EXP: return rnd(dt, "expf(" + a + ")");
    case FGT_OP_LOG: return rnd(dt, "logf(" + a + ")");
    case FGT_OP_SQRT: return rnd(dt, "__fsqrt_rn(" + a + ")");
    case FGT_OP_SIN: return rnd(dt, "sinf(" + a + ")");
    case FGT_OP_COS: return rnd(dt, "cosf(" + a + ")");
    case FGT_OP_TANH: return rnd(dt, "tanhf(" + a + ")");
    case FGT_OP_ERF: return rnd(dt, "erff(" + a + ")");
    case FGT_OP_FLOOR: return "floorf(" + a + ")";
    case FGT_OP_CEIL: return "ceilf(" + a + ")";
    case FGT_OP_ROUND: return "rintf(" + a + ")";
    case FGT_OP_ABS:
      if (is_float(dt)) return "fabsf(" + a + ")";
      return "((" + a + ")<0?(" + vt_t(dt) + ")((" + ut_t(dt) + ")0-(" + ut_t(dt) + ")(" + a + ")):(" + a + "))";
    case FGT_OP_BITWISE_NOT: return dt == FGT_BOOL ? "(!" + a + ")" : "(~" + a + ")";
  }
  fail(FGT_ERR_UNSUPPORTED, "unary opcode not supported by the generator");
}

bool expensive(int op) {
  switch (op) {
    case FGT_OP_EXP:
    case FGT_OP_LOG:
    case FGT_OP_SQRT:
    case FGT_OP_SIN:
    case FGT_OP_COS:
    case FGT_OP_TANH:
    case FGT_OP_ERF:
    case FGT_OP_POW:
      return true;
  }
  return false;
}

// ----------------------------------------------------- reduction algebra ---
enum Ctx { CTX_ROW, CTX_COL, CTX_FULL, CTX_FIN };

struct RedText {
  bool arg = false, is_max = false, fl = false;
  std::string acc_t, part_t, fin_t, ident, identi;
  int op = 0, dt = 0, odt = 0;  // reduction op, result dtype, operand dtype
  bool storage = false;
};

RedText red_text(const Graph& g, int node, int policy, Ctx ctx) {
  const Node& n = g.nodes[node];
  const Node& x = g.nodes[n.args[0]];
  RedText t;
  t.op = n.op;
  t.dt = n.dt;
  t.odt = x.dt;
  t.fl = is_float(x.dt);
  t.storage = policy == FGT_ACCUM_STORAGE;
  if (is_argreduce(n.op)) {
    t.arg = true;
    t.is_max = n.op == FGT_OP_ARGMAX;
    t.acc_t = t.part_t = t.fin_t = vt_t(x.dt);
    if (t.fl) t.ident = t.is_max ? "__int_as_float(0xff800000)" : "__int_as_float(0x7f800000)";
    else t.ident = t.is_max ? min_lit(x.dt) : max_lit(x.dt);
    t.identi = "9223372036854775807LL";
    return t;
  }
  switch (n.op) {
    case FGT_OP_REDUCE_SUM:
    case FGT_OP_REDUCE_PROD: {
      std::string one = n.op == FGT_OP_REDUCE_SUM ? "0" : "1";
      if (t.fl && !t.storage) {
        // f32 within a thread's bounded span (a row, or a CTA's rows of one
        // column), f64 across unbounded spans (grid-stride loops, partials).
        t.acc_t = (ctx == CTX_FULL || ctx == CTX_FIN) ? "double" : "float";
        t.part_t = ctx == CTX_COL ? "float" : "double";
        t.fin_t = "double";
        t.ident = (ctx == CTX_FULL || ctx == CTX_FIN) ? one + ".0" : one + ".0f";
      } else if (t.fl) {
        t.acc_t = t.part_t = t.fin_t = "float";
        t.ident = one + ".0f";
      } else {
        t.acc_t = t.part_t = t.fin_t = vt_t(x.dt);
        t.ident = "((" + vt_t(x.dt) + ")" + one + ")";
      }
      break;
    }
    case FGT_OP_REDUCE_MAX:
    case FGT_OP_REDUCE_MIN: {
      bool mx = n.op == FGT_OP_REDUCE_MAX;
      t.acc_t = t.part_t = t.fin_t = vt_t(x.dt);
      if (t.fl) t.ident = mx ? "__int_as_float(0xff800000)" : "__int_as_float(0x7f800000)";
      else t.ident = mx ? min_lit(x.dt) : max_lit(x.dt);
      break;
    }
    case FGT_OP_REDUCE_ANY:
    case FGT_OP_REDUCE_ALL:
      t.acc_t = t.fin_t = "bool";
      t.part_t = "fgt_u8";
      t.ident = n.op == FGT_OP_REDUCE_ANY ? "false" : "true";
      break;
  }
  return t;
}

// a = a (+) b for a value reduction, as a statement.
std::string comb_stmt(const RedText& t, const std::string& a, const std::string& b) {
  const std::string T = vt_t(t.odt), U = ut_t(t.odt);
  switch (t.op) {
    case FGT_OP_REDUCE_SUM:
      if (t.fl) return a + " = " + (t.storage ? rnd(t.odt, "__fadd_rn(" + a + "," + b + ")") : a + " + " + b) + ";";
      return a + " = fgt_wrap_add<" + T + "," + U + ">(" + a + "," + b + ");";
    case FGT_OP_REDUCE_PROD:
      if (t.fl) return a + " = " + (t.storage ? rnd(t.odt, "__fmul_rn(" + a + "," + b + ")") : a + " * " + b) + ";";
      return a + " = fgt_wrap_mul<" + T + "," + U + ">(" + a + "," + b + ");";
    case FGT_OP_REDUCE_MAX:
      return a + " = " + (t.fl ? "fgt_fmax(" : "fgt_imax<" + T + ">(") + a + "," + b + ");";
    case FGT_OP_REDUCE_MIN:
      return a + " = " + (t.fl ? "fgt_fmin(" : "fgt_imin<" + T + ">(") + a + "," + b + ");";
    case FGT_OP_REDUCE_ANY: return a + " = " + a + " || " + b + ";";
    case FGT_OP_REDUCE_ALL: return a + " = " + a + " && " + b + ";";
  }
  return "";
}
std::string arg_stmt(const RedText& t, const std::string& a, const std::string& ai, const std::string& b,
                     const std::string& bi) {
  std::string fn = t.fl ? std::string("fgt_arg_better_f<") + (t.is_max ? "true" : "false") + ">"
                        : std::string("fgt_arg_better_i<") + (t.is_max ? "true" : "false") + "," + vt_t(t.odt) + ">";
  return "if (" + fn + "(" + b + "," + bi + "," + a + "," + ai + ")) { " + a + " = " + b + "; " + ai + " = " + bi + "; }";
}
// Argmax/argmin update for a thread scanning its elements in increasing
// index order (ties keep the earlier element without comparing indices).
std::string scan_stmt(const RedText& t, const std::string& a, const std::string& ai, const std::string& b,
                      const std::string& bi) {
  std::string fn = t.fl ? std::string("fgt_arg_scan_f<") + (t.is_max ? "true" : "false") + ">"
                        : std::string("fgt_arg_scan_i<") + (t.is_max ? "true" : "false") + "," + vt_t(t.odt) + ">";
  // lane-local indices are int (sentinel INT_MAX), others int64 (INT64_MAX)
  const bool local = bi == "v";
  const std::string unset = local ? "0x7fffffff" : "9223372036854775807LL";
  return "if (" + fn + "(" + b + "," + a + "," + ai + "," + unset + ")) { " + a + " = " + b + "; " + ai + " = " + bi + "; }";
}

// Round a finished accumulator to the reduction's result dtype (once).
std::string finalize(const RedText& t, const std::string& acc, const std::string& acc_t) {
  if (!t.fl || t.op == FGT_OP_REDUCE_MAX || t.op == FGT_OP_REDUCE_MIN) return acc;
  if (acc_t == "double") {
    if (t.dt == FGT_F32) return "__double2float_rn(" + acc + ")";
    if (t.dt == FGT_F16) return "fgt_rnd_f16(fgt_f64_to_f32_odd(" + acc + "))";
    return "fgt_rnd_bf16(fgt_f64_to_f32_odd(" + acc + "))";
  }
  return rnd(t.dt, acc);
}

// ------------------------------------------------------------------ emitter -
enum ScKind { SC_PRO, SC_PROLANE, SC_ROW, SC_LANE, SC_CACHE };
struct Sc {
  ScKind k;
  int p;
};

struct Emitter {
  const Plan& P;
  const Graph& g;
  const KernelDef& K;
  int row_phases = 0;  // levels holding row reductions (one block barrier each per row)
  bool parity_rows = false;  // row reductions alternate two partial buffers (it_ counts rows)
  std::vector<std::string> rowpf, rowpf_first, rowpf_next;  // row-scope loads, one row ahead
  std::map<std::string, std::pair<std::string, Sc>> unrounded;  // bf16 temp -> (f32 expression, scope)
  std::map<std::string, std::string> texpr;  // temp -> its defining expression
  std::map<std::string, std::string> cse;    // (scope, type, expression) -> temp
  std::set<int> div_phases;                 // phases with element divisions by a hoisted reciprocal
  std::map<int, std::set<std::string>> div_rcps;  // the reciprocals those divisions use, per phase
  std::set<int> exp_phases;                 // phases with element exps by fgt_exp_q (range noted)
  std::set<int> col_phases;                 // phases updating column accumulators (not redoable)
  std::vector<std::string> llpre;           // peer-exchange FIN: record words requested before they are combined
  std::set<int> tm_phases;                  // phases updating column accumulators held in TMEM
  int64_t tm_alloc = 0;                     // TMEM columns allocated per CTA (0: none)
  std::map<int, std::vector<std::string>> resets;  // row accumulators of a phase back to identity
  std::set<std::string> f32_sum_accs;       // f32 sum accumulators (arrays) whose two lanes may add as a pair
  int64_t col_smem = 0;                     // bytes of column accumulators in shared memory (before the ring)
  const Domain& d;
  std::set<int64_t>* temps_loaded;
  std::vector<RedDef> fin_reds;
  Analyzer an;
  bool row = false, elem = false, fin = false, cached = false;
  int nphase = 1;
  int U = 1;

  std::vector<std::string> kdecl, prosites, prolane, rowdecl, rowend, kend;
  // Streamed operands of a register-resident row: loaded for the next row
  // while the current one is computed (software pipelining across rows).
  struct RowSite {
    std::string name, st, ptr;
    Idx addr;      // contiguous: row base (element part zero); uniform: full address
    bool uniform;
    int bytes = 0;         // one thread's piece per chunk (VEC elements)
    bool staged = false;   // copied through the shared-memory stage ring
    bool packed = false;   // 16-bit values two per 32-bit word ([NCH][VEC / 2] words)
    int64_t smem_off = 0;  // region of this operand in the ring
  };
  std::vector<RowSite> row_sites;
  // per-thread column operands persisted in registers (name, words per chunk)
  std::vector<std::pair<std::string, int>> persisted_arrays;
  // Ring-resident rows (FGT_ROW_RING_RESIDENT): a staged operand's current row
  // stays in its ring stage, and each phase that reads it copies the thread's
  // own pieces of the chunk into a phase-local array (the name maps to the
  // operand's index in row_sites).
  std::map<std::string, int> resident_loc;
  bool resident() const { return P.opt.ring_resident && cached && K.cluster == 1; }
  // Narrow division applies when every floating output of the partition is
  // f16 / bf16: their rounding hides the product's at most one-ulp f32 error.
  bool narrow_div() const {
    if (!P.opt.narrow_div) return false;
    for (int o : g.outputs) {
      const int dt = g.nodes[o].dt;
      if (is_float(dt) && dtype_size(dt) != 2) return false;
    }
    return true;
  }
  int stages = 0;                  // shared-memory ring depth (0: register path)
  int64_t stage_bytes = 0;         // bytes of one stage (all staged operands)
  // Shared-memory address (bytes from the dynamic base) of a thread's piece.
  std::string piece_off(const RowSite& rs, const std::string& stg) {
    // a thread's own piece within this CTA (in a cluster the CTA holds
    // nt of the row's tpr threads: index by the CTA-local thread)
    const bool cl = K.cluster > 1;
    return "(" + std::to_string(rs.smem_off) + "u + (unsigned)((((" + stg + ") * " + std::to_string(K.rows_per_cta) +
           " + grp) * " + std::to_string(K.nch) + " + c) * " + std::to_string(cl ? K.nt : K.tpr) + " + " +
           (cl ? "tid" : "lane") + ") * " + std::to_string(rs.bytes) + "u)";
  }
  std::string site_load(const RowSite& rs, const std::string& arr, const char* rvar) {
    if (rs.uniform) return arr + "[c] = " + rs.ptr + "[" + itext(rs.addr, "e0", rvar) + "];";
    if (rs.packed) return "fgt_vload(" + arr + "[c], (const fgt_u32*)(" + rs.ptr + " + " + itext(rs.addr, "e", rvar) + " + e0));";
    return "fgt_vload(" + arr + "[c], " + rs.ptr + " + " + itext(rs.addr, "e", rvar) + " + e0);";
  }
  std::vector<std::vector<std::string>> rowsc, lane, chunkpre, chunkpost, post;
  std::vector<std::string> eload;  // ELEM: site loads (per u)
  std::map<std::string, std::string> memo;
  std::map<int, std::string> red_var;  // node -> variable holding its value
  int uid = 0;

  Emitter(const Plan& P_, const KernelDef& K_, std::set<int64_t>* tl)
      : P(P_), g(P_.g), K(K_), d(K_.dom), temps_loaded(tl), an(P_.g, P_.loc, K_.kind, K_.dom) {
    row = K.kind == KKind::ROW;
    elem = K.kind == KKind::ELEM;
    fin = K.kind == KKind::COLFIN || K.kind == KKind::FULLFIN;
    cached = row && !K.streaming;
    U = elem ? K.unroll : 1;
    fin_reds = K.reds;
    for (auto& rd : fin_reds) an.group[rd.node] = &rd;
    if (K.scatter_stage == 3) an.finalize_scatter = K.scatter_node;
  }

  std::string fresh(const char* p) { return std::string(p) + std::to_string(uid++); }
  bool pairs() const { return P.opt.lane_pairs && K.vec % 2 == 0; }
  // 16-bit operands held two per 32-bit register (element v of a chunk is
  // half v % 2 of word v / 2): half the registers of one value per register
  bool pack16(int dt) const { return P.opt.lane_pairs && K.vec % 2 == 0 && dtype_size(dt) == 2; }

  void add(Sc s, const std::string& st) {
    switch (s.k) {
      case SC_PRO: kdecl.push_back(st); break;
      case SC_PROLANE: prolane.push_back(st); break;
      case SC_ROW: rowsc[s.p].push_back(st); break;
      default: lane[s.p].push_back(st); break;
    }
  }

  // Integer index text in the given scope. Digits collapse to r / e when the
  // coefficients follow the mixed radix (the common, vectorisable case).
  // evar / rvar name the element and row linear indices the text is for; the
  // digit variables o<k>/i<k> exist only for the current row and element, so
  // other names get their digits by division.
  std::string itext(const Idx& a, const char* evar = "e", const char* rvar = "r") {
    if (!a.aff) return "(" + a.code + ")";
    std::ostringstream s;
    s << "(" << a.k << "LL";
    bool prop = d.no() > 0;
    int64_t alpha = d.no() ? a.c[d.no() - 1] : 0;
    for (int k = 0; k < d.no() && prop; ++k)
      if (a.c[k] != alpha * d.ow[k]) prop = false;
    if (prop) {
      if (alpha) s << "+" << alpha << "LL*" << rvar;
    } else {
      for (int k = 0; k < d.no(); ++k) {
        if (!a.c[k]) continue;
        if (std::string(rvar) == "r") s << "+" << a.c[k] << "LL*o" << k;
        else s << "+" << a.c[k] << "LL*((" << rvar << "/" << d.ow[k] << "LL)%" << d.od[k] << "LL)";
      }
    }
    const int ni = (int)d.id.size();
    bool propi = ni > 0;
    int64_t beta = ni ? a.c[d.no() + ni - 1] : 0;
    for (int k = 0; k < ni && propi; ++k)
      if (a.c[d.no() + k] != beta * d.iw[k]) propi = false;
    if (propi) {
      if (beta) s << "+" << beta << "LL*" << evar;
    } else {
      for (int k = 0; k < ni; ++k) {
        if (!a.c[d.no() + k]) continue;
        if (std::string(evar) == "e") s << "+" << a.c[d.no() + k] << "LL*i" << k;
        else s << "+" << a.c[d.no() + k] << "LL*((" << evar << "/" << d.iw[k] << "LL)%" << d.id[k] << "LL)";
      }
    }
    s << ")";
    return s.str();
  }

  // Is the affine address exactly base(o) + e with base aligned to the vector?
  bool contiguous(const Idx& a, std::string* base) {
    if (!a.aff || d.id.empty()) return false;
    for (int k = 0; k < (int)d.id.size(); ++k)
      if (a.c[d.no() + k] != d.iw[k]) return false;
    if (d.NI % K.vec) return false;
    if (a.k % K.vec) return false;
    for (int k = 0; k < d.no(); ++k)
      if (a.c[k] % K.vec) return false;
    Idx b = a;
    for (int k = 0; k < (int)d.id.size(); ++k) b.c[d.no() + k] = 0;
    *base = itext(b);
    return true;
  }
  bool uniform(const Idx& a) {
    if (!a.aff || d.id.empty()) return false;
    if (a.c[d.nd() - 1] != 0) return false;
    return d.id.back() % K.vec == 0;
  }

  std::string ptr_of(int node, bool for_store = false, int port = -1, int64_t temp = -1) {
    const Node& n = g.nodes[node];
    const std::string T = st_t(n.dt);
    if (for_store) {
      if (port >= 0) return "((" + T + "*)p.out[" + std::to_string(port) + "])";
      return "((" + T + "*)(p.ws+" + std::to_string(temp) + "LL))";
    }
    const Loc& L = P.loc[node];
    if (L.kind == Loc::INPUT) return "((const " + T + "*)p.in[" + std::to_string(L.index) + "])";
    if (L.kind == Loc::OUTPUT) return "((const " + T + "*)p.out[" + std::to_string(L.index) + "])";
    if (temps_loaded) temps_loaded->insert(L.offset);
    return "((const " + T + "*)(p.ws+" + std::to_string(L.offset) + "LL))";
  }

  // Phase p's copy of staged operand row_sites[idx] for the current chunk:
  // read from the current row's ring stage at the top of the chunk (the
  // stage offset is resolved when the ring is laid out: @PIECE<idx>@).
  std::string resident_local(int idx, int p) {
    const RowSite& rs = row_sites[idx];
    const std::string key = "rloc|" + rs.name + "|" + std::to_string(p);
    auto it = memo.find(key);
    if (it != memo.end()) return it->second;
    const std::string loc = fresh("rs");
    memo[key] = loc;
    resident_loc[loc] = idx;
    const std::string W = std::to_string(rs.packed ? K.vec / 2 : K.vec);
    chunkpre[p].push_back(rs.st + " " + loc + "[" + W + "]; fgt_lds(" + loc + ", (const " + rs.st + "*)(fgt_dsmem + @PIECE" +
                          std::to_string(idx) + "@));");
    return loc;
  }

  std::string load(int id, const Map& m, Sc D) {
    const Node& n = g.nodes[id];
    Idx A = to_linear(m, n.shape, d);
    const std::string ptr = ptr_of(id);
    const std::string VT = vt_t(n.dt), ST = st_t(n.dt);
    if (!m.guard.empty()) {
      // below pad / concatenate / gather: read only where the guard holds
      std::string v = fresh("x");
      add(D, "const " + VT + " " + v + " = (" + m.guard + ") ? " + ld_conv(n.dt, "__ldg(" + ptr + " + " + itext(A) + ")") +
                 " : (" + VT + ")0;");
      return v;
    }
    if (D.k == SC_PRO) {
      std::string v = fresh("g");
      add(D, "const " + VT + " " + v + " = " + ld_conv(n.dt, ptr + "[" + itext(A) + "]") + ";");
      return v;
    }
    if (D.k == SC_ROW) {
      std::string v = fresh("w");
      if (row && cached) {
        // Loaded one row ahead: the raw value of row r+stride is requested
        // while row r is computed, and converted when that row starts.
        const std::string pf = v + "_pf";
        kdecl.push_back(ST + " " + pf + " = (" + ST + ")0;");
        const std::string ld = pf + " = rv ? " + ptr + "[" + itext(A) + "] : (" + ST + ")0;";
        rowpf_first.push_back(ld);
        rowpf_next.push_back(ld);
        rowpf.push_back("const " + VT + " " + v + " = " + ld_conv(n.dt, pf) + ";");
        return v;
      }
      add(D, "const " + VT + " " + v + " = rv ? " + ld_conv(n.dt, ptr + "[" + itext(A) + "]") + " : (" + VT + ")0;");
      return v;
    }
    std::string base;
    const bool prol = D.k == SC_PROLANE;
    std::string ctx = prol ? "P" : cached ? "R" : elem ? "E" : ("S" + std::to_string(D.p));
    if (contiguous(A, &base)) {
      std::string key = "site" + ctx + "|" + std::to_string(id) + "|" + base;
      auto it = memo.find(key);
      std::string s;
      if (it != memo.end()) s = it->second;
      else {
        s = fresh("s");
        memo[key] = s;
        const bool pk = pack16(n.dt);
        const std::string vec = std::to_string(pk ? K.vec / 2 : K.vec), SS = pk ? std::string("fgt_u32") : ST;
        const std::string src = pk ? "(const fgt_u32*)(" + ptr + " + " + base + " + e0)" : ptr + " + " + base + " + e0";
        if (prol) {
          prosites.push_back(SS + " " + s + "[" + vec + "]; fgt_vload_keep(" + s + ", " + src + ");");
        } else if (cached) {
          Idx b = A;
          for (int k = 0; k < (int)d.id.size(); ++k) b.c[d.no() + k] = 0;
          RowSite rs{s, SS, ptr, b, false};
          rs.packed = pk;
          rs.bytes = K.vec * dtype_size(n.dt);
          // cp.async moves 4, 8 or 16 bytes; a stage (one row of every staged
          // operand) must fit the ring budget.
          const int64_t piece = (int64_t)K.rows_per_cta * K.nch * (K.tpr / K.cluster) * rs.bytes;
          // ring-resident rows need two stages: the current row and the next
          const int64_t budget = (int64_t)P.opt.ring_kb * 1024 / (resident() ? 2 : 1);
          rs.staged = P.opt.row_staging && (rs.bytes == 4 || rs.bytes == 8 || rs.bytes == 16) &&
                      stage_bytes + piece <= budget;
          if (rs.staged) stage_bytes += piece;
          row_sites.push_back(rs);
        } else if (elem) {
          eload.push_back("fgt_vload(" + s + "[u], " + src + ");");
          rowdecl.push_back(SS + " " + s + "[" + std::to_string(U) + "][" + vec + "];");
        } else {
          chunkpre[D.p].push_back(SS + " " + s + "[" + vec + "]; fgt_vload(" + s + ", " + src + ");");
        }
      }
      std::string arr = prol ? s : cached ? s + "[c]" : elem ? s + "[u]" : s;
      if (cached && !prol && resident()) {
        int idx = -1;
        for (size_t k = 0; k < row_sites.size(); ++k)
          if (row_sites[k].name == s) idx = (int)k;
        if (idx >= 0 && row_sites[idx].staged) arr = resident_local(idx, D.k == SC_LANE ? D.p : 0);
      }
      if (pack16(n.dt)) return ld_conv(n.dt, "fgt_h16(" + arr + ", v)");
      return ld_conv(n.dt, arr + "[v]");
    }
    if (uniform(A)) {
      std::string at = itext(A, "e0");
      std::string key = "uni" + ctx + "|" + std::to_string(id) + "|" + at;
      auto it = memo.find(key);
      std::string s;
      if (it != memo.end()) s = it->second;
      else {
        s = fresh("u");
        memo[key] = s;
        if (prol) prosites.push_back("const " + ST + " " + s + " = " + ptr + "[" + at + "];");
        else if (cached) {
          row_sites.push_back(RowSite{s, ST, ptr, A, true});
        } else if (elem) {
          rowdecl.push_back(ST + " " + s + "[" + std::to_string(U) + "];");
          eload.push_back(s + "[u] = " + ptr + "[" + at + "];");
        } else {
          chunkpre[D.p].push_back("const " + ST + " " + s + " = " + ptr + "[" + at + "];");
        }
      }
      if (prol) return ld_conv(n.dt, s);
      if (cached) return ld_conv(n.dt, s + "[c]");
      if (elem) return ld_conv(n.dt, s + "[u]");
      return ld_conv(n.dt, s);
    }
    std::string v = fresh("x");
    add(D, "const " + VT + " " + v + " = " + ld_conv(n.dt, "__ldg(" + ptr + " + " + itext(A) + ")") + ";");
    return v;
  }

  // Value of node `id` read at map m, usable from scope s.
  std::string val(int id, const Map& m, Sc s) {
    Level L = an.run(id, m);
    Sc D{SC_PRO, 0};
    if (L.kind == 0) D = {SC_PRO, 0};
    else if (L.kind == 1) D = {SC_ROW, L.phase};
    else if (L.kind == 2) D = cached ? Sc{SC_PROLANE, 0} : Sc{SC_LANE, s.k == SC_LANE ? s.p : 0};
    else {
      require(s.k == SC_LANE, "internal: element value requested outside an element loop", FGT_ERR_UNSUPPORTED);
      D = {SC_LANE, s.p};
      if (cached && s.p > L.phase && expensive(g.nodes[id].op) && m.guard.empty()) D = {SC_CACHE, L.phase};
    }
    if (s.k == SC_PROLANE && D.k == SC_LANE) D = s;
    // a prologue value read from the row loop goes through its persisted
    // register copy, keyed apart from the prologue-local temporary
    const bool persisted = D.k == SC_PROLANE && s.k != SC_PROLANE;
    std::string key = std::to_string(id) + "@" + m.key() + "#" + std::to_string((int)D.k) + ":" +
                      std::to_string(D.p) + (persisted ? "+cv" : "");
    auto it = memo.find(key);
    if (it != memo.end()) return it->second;
    std::string r;
    const Node& n = g.nodes[id];
    if (D.k == SC_CACHE) {
      std::string v = val(id, m, Sc{SC_LANE, D.p});
      std::string cname = fresh("c");
      rowdecl.push_back(vt_t(n.dt) + " " + cname + "[" + std::to_string(K.nch) + "][" + std::to_string(K.vec) + "];");
      lane[D.p].push_back(cname + "[c][v] = " + v + ";");
      r = cname + "[c][v]";
    } else if (persisted) {
      std::string v = val(id, m, Sc{SC_PROLANE, 0});
      std::string cname = fresh("cv");
      if ((resident() || P.opt.pack_cols) && pack16(n.dt)) {
        // a 16-bit value is exact in its storage bits: two per register
        kdecl.push_back("fgt_u32 " + cname + "[" + std::to_string(K.nch) + "][" + std::to_string(K.vec / 2) + "];");
        prolane.push_back("fgt_set_h16(" + cname + "[c], v, " + st_conv(n.dt, v) + ");");
        r = ld_conv(n.dt, "fgt_h16(" + cname + "[c], v)");
        persisted_arrays.push_back({cname, K.vec / 2});
      } else {
        kdecl.push_back(vt_t(n.dt) + " " + cname + "[" + std::to_string(K.nch) + "][" + std::to_string(K.vec) + "];");
        prolane.push_back(cname + "[c][v] = " + v + ";");
        r = cname + "[c][v]";
        persisted_arrays.push_back({cname, K.vec});
      }
      memo[key] = r;
      return r;
    } else {
      r = define(id, m, D);
    }
    memo[key] = r;
    return r;
  }

  std::string define(int id, const Map& m, Sc D) {
    const Node& n = g.nodes[id];
    auto rv = red_var.find(id);
    if (rv != red_var.end() && an.group.count(id)) return rv->second;
    const bool completes = id == K.scatter_node && K.scatter_stage == 3;
    if (P.loc[id].kind != Loc::NONE && !an.group.count(id) && !completes) return load(id, m, D);
    switch (n.op) {
      case FGT_OP_CONSTANT:
        return literal(n.dt, n.cbits);
      case FGT_OP_IOTA: {
        auto C = to_coords(m, n.shape, d);
        std::string t = itext(C[n.attrs[0]]);
        auto io = P.iota_offsets.find(id);
        if (io != P.iota_offsets.end()) t = "(" + t + "+" + std::to_string(io->second) + "LL)";
        return cast_expr(FGT_I64, n.dt, t);
      }
      case FGT_OP_SPLAT:
      case FGT_OP_RESHAPE:
      case FGT_OP_BROADCAST_IN_DIM:
      case FGT_OP_TRANSPOSE:
      case FGT_OP_SLICE:
      case FGT_OP_STOP_GRADIENT: {
        auto ms = operand_maps(g, id, m, d);
        return val(n.args[0], ms[0], D);
      }
      case FGT_OP_PAD: {
        auto ms = operand_maps(g, id, m, d);
        const std::string xv = val(n.args[0], ms[0], D), pv = val(n.args[1], ms[1], D);
        const std::string cond = pad_condition(g, id, m, d);
        if (cond.empty()) return xv;
        std::string v = fresh("t");
        add(D, "const " + vt_t(n.dt) + " " + v + " = (" + cond + ") ? " + xv + " : " + pv + ";");
        return v;
      }
      case FGT_OP_CONCATENATE: {
        auto ms = operand_maps(g, id, m, d);
        const std::string av = val(n.args[0], ms[0], D), bv = val(n.args[1], ms[1], D);
        std::string v = fresh("t");
        add(D, "const " + vt_t(n.dt) + " " + v + " = (" + concat_condition(g, id, m, d) + ") ? " + av + " : " + bv + ";");
        return v;
      }
      case FGT_OP_SCATTER_ADD: {
        // the kernel that completes the scatter: base + accumulator, one
        // rounding to the dtype (integers wrap)
        require(id == K.scatter_node && K.scatter_stage == 3, "internal: scatter_add read before it is complete",
                FGT_ERR_UNSUPPORTED);
        const std::string bv = val(n.args[0], m, D);
        std::string av = scatter_acc_ptr() + "[" + itext(to_linear(m, n.shape, d)) + "]";
        if (K.scatter_csr) {
          // this element's row bucket: the update rows scattered to it, each
          // read once by pointer, summed in the accumulator type
          const Node& up = g.nodes[n.args[2]];
          const int64_t HN = n.n() / n.shape[0];
          const std::string H = std::to_string(HN) + "LL";
          const std::string NUS = std::to_string(std::max<int64_t>(1, g.nodes[n.args[1]].n())) + "LL";
          const std::string A = csr_acc_t();
          const Idx li = to_linear(m, n.shape, d);
          const std::string lin = itext(li);
          // the element's linear index is the kernel's element index e (the
          // base's own row-major order): a chunk is VEC consecutive elements
          bool ident = li.aff && li.k == 0 && (int)li.c.size() == d.nd();
          for (int j = 0; ident && j < d.nd(); ++j) ident = li.c[j] == d.iw[j];
          if (elem && D.k == SC_LANE && ident && n.n() == d.NI && HN % K.vec == 0) {
            // a chunk's VEC elements share one row: walk its list once and
            // read VEC consecutive update values per entry, two entries per
            // step (the second entry's loads issue before the first's values
            // are summed); at most NU hops
            auto it = memo.find("csr_chunk");
            std::string sa;
            if (it != memo.end()) sa = it->second;
            else {
              sa = fresh("sa");
              memo["csr_chunk"] = sa;
              const std::string V = std::to_string(K.vec), ST = st_t(up.dt), U = ptr_of(n.args[2]);
              const std::string add_a = "for (int v = 0; v < " + V + "; ++v) " + sa + "[v] += (" + A + ")(" + ld_conv(up.dt, "ua_[v]") + ");";
              const std::string add_b = "for (int v = 0; v < " + V + "; ++v) " + sa + "[v] += (" + A + ")(" + ld_conv(up.dt, "ub_[v]") + ");";
              chunkpre[0].push_back(
                  A + " " + sa + "[" + V + "]; for (int v = 0; v < " + V + "; ++v) " + sa + "[v] = 0; { const fgt_i64 r_ = e0 / " + H +
                  ", h_ = e0 - r_ * " + H + "; int i_ = " + ll_head() + "[r_]; for (fgt_i64 n_ = 0; i_ >= 0 && n_ < " + NUS +
                  "; n_ += 2) { " + ST + " ua_[" + V + "]; fgt_vload_keep(ua_, " + U + " + (fgt_i64)i_ * " + H + " + h_); const int j_ = " +
                  ll_next() + "[i_]; if (j_ >= 0) { " + ST + " ub_[" + V + "]; fgt_vload_keep(ub_, " + U + " + (fgt_i64)j_ * " + H +
                  " + h_); const int k_ = " + ll_next() + "[j_]; " + add_a + " " + add_b + " i_ = k_; } else { " + add_a +
                  " i_ = -1; } } }");
            }
            av = sa + "[v]";
          } else {
            av = fresh("sa");
            add(D, A + " " + av + " = 0; { const fgt_i64 l_ = " + lin + "; const fgt_i64 r_ = l_ / " + H + ", h_ = l_ - r_ * " + H +
                       "; int i_ = " + ll_head() + "[r_]; for (fgt_i64 n_ = 0; i_ >= 0 && n_ < " + NUS + "; ++n_) { " + av +
                       " += (" + A + ")(" + ld_conv(up.dt, ptr_of(n.args[2]) + "[(fgt_i64)i_ * " + H + " + h_]") + "); i_ = " +
                       ll_next() + "[i_]; } }");
          }
        }
        std::string expr;
        if (n.dt == FGT_F32) expr = "__double2float_rn((double)" + bv + " + " + av + ")";
        else if (is_float(n.dt)) expr = rnd(n.dt, "fgt_f64_to_f32_odd((double)" + bv + " + " + av + ")");
        else expr = "fgt_wrap_add<" + vt_t(n.dt) + "," + ut_t(n.dt) + ">(" + bv + ", (" + vt_t(n.dt) + ")" + av + ")";
        std::string v = fresh("t");
        add(D, "const " + vt_t(n.dt) + " " + v + " = " + expr + ";");
        return v;
      }
      case FGT_OP_GATHER: {
        auto ms = operand_maps(g, id, m, d);
        const std::string gx = gather_index_name(id, m);
        const std::string iv = val(n.args[1], ms[1], D);
        add(D, "const fgt_i64 " + gx + " = (fgt_i64)(" + iv + ");");
        const std::string pv = val(n.args[0], ms[0], D);
        std::string v = fresh("t");
        add(D, "const " + vt_t(n.dt) + " " + v + " = (" + gx + ">=0LL&&" + gx + "<" +
                   std::to_string(g.nodes[n.args[0]].shape[n.attrs[0]]) + "LL) ? " + pv + " : (" + vt_t(n.dt) + ")0;");
        return v;
      }
      default:
        break;
    }
    auto ms = operand_maps(g, id, m, d);
    std::vector<std::string> a;
    for (size_t k = 0; k < n.args.size(); ++k) a.push_back(val(n.args[k], ms[k], D));
    std::string expr;
    const int odt = g.nodes[n.args[0]].dt;
    if (n.op == FGT_OP_DIV) {
      // A divisor that is constant across the row's elements (a row statistic
      // or a kernel constant) gets its reciprocal once, in its own scope; the
      // per-element division is then the corrected reciprocal product, which
      // equals the IEEE quotient (fgt_div_by).
      const Level la = an.run(n.args[0], ms[0]), lb = an.run(n.args[1], ms[1]);
      unsigned dbits = 0;
      const bool pow2 = std::sscanf(a[1].c_str(), "__uint_as_float(0x%8xu)", &dbits) == 1 && (dbits & 0x7fffffu) == 0 &&
                        ((dbits >> 23) & 0xffu) >= 1 && ((dbits >> 23) & 0xffu) <= 253;
      if (!pow2 && (lb.kind & 2) == 0 && (la.kind & 2) != 0) {
        const Sc db = lb.kind == 0 ? Sc{SC_PRO, 0} : Sc{SC_ROW, lb.phase};
        const std::string rk = "rcp|" + a[1] + "#" + std::to_string((int)db.k) + ":" + std::to_string(db.p);
        auto it = memo.find(rk);
        std::string rcp;
        if (it != memo.end()) rcp = it->second;
        else {
          rcp = fresh("rcp");
          memo[rk] = rcp;
          add(db, "const float " + rcp + " = fgt_recip_for_div(" + a[1] + ");");
        }
        if (D.k == SC_LANE) {
          // Per element: the corrected reciprocal product, and a note of |q|
          // in the phase's range trackers. The phase is redone with IEEE
          // division by any thread whose trackers leave the range where the
          // product is exact (see the phase assembly in build_row); kernels
          // that cannot redo a phase get the per-element guarded form.
          const std::string q = fresh("q");
          add(D, "const float " + q + " = @DIVQ@(" + a[0] + "," + a[1] + "," + rcp + ");");
          add(D, "@NOTE@(" + q + ");");
          div_phases.insert(D.p);
          div_rcps[D.p].insert(rcp);
          expr = rnd(n.dt, q);
        } else {
          expr = rnd(n.dt, "fgt_div_by(" + a[0] + "," + a[1] + "," + rcp + ")");
        }
      }
    }
    if (expr.empty() && n.op == FGT_OP_EXP && is_float(n.dt) && D.k == SC_LANE && row && cached && P.opt.own_exp) {
      // e^x by fgt_exp_q with a note of |x|: the phase is redone with expf by
      // any thread whose arguments left |x| <= 86 (or held a NaN / inf)
      const std::string x = fresh("xe");
      add(D, "const float " + x + " = @EXPQ@(" + a[0] + ");");
      add(D, "@ENOTE@(" + a[0] + ");");
      exp_phases.insert(D.p);
      expr = rnd(n.dt, x);
    }
    if (!expr.empty()) {
    } else if (n.op == FGT_OP_CAST) expr = cast_expr(odt, n.dt, a[0]);
    else if (n.op == FGT_OP_COMPARE) expr = "(" + a[0] + cmp_op(n.pred) + a[1] + ")";
    else if (n.op == FGT_OP_SELECT) expr = "(" + a[0] + "?" + a[1] + ":" + a[2] + ")";
    else if (is_binary(n.op)) expr = binary_expr(n.op, n.dt, a[0], a[1]);
    else if (is_unary(n.op)) expr = unary_expr(n.op, n.dt, a[0]);
    else fail(FGT_ERR_UNSUPPORTED, std::string("generator cannot place ") + opcode_name(n.op));
    // Identical pure expressions in one scope share one temporary (graph
    // nodes that differ only in shape, e.g. [R] and [R, 1] row statistics,
    // produce the same text).
    const std::string ck = std::to_string((int)D.k) + ":" + std::to_string(D.p) + "|" + vt_t(n.dt) + "|" + expr;
    auto hit = cse.find(ck);
    if (hit != cse.end()) return hit->second;
    std::string v = fresh("t");
    add(D, "const " + vt_t(n.dt) + " " + v + " = " + expr + ";");
    cse[ck] = v;
    texpr[v] = expr;
    // A bf16 value is the rounding of an f32 expression; a store of it may
    // round pairs at once instead (store_stmt_elem).
    static const std::string kRnd = "fgt_rnd_bf16(";
    if (n.dt == FGT_BF16 && expr.compare(0, kRnd.size(), kRnd) == 0 && expr.back() == ')')
      unrounded[v] = {expr.substr(kRnd.size(), expr.size() - kRnd.size() - 1), D};
    return v;
  }

  // ---------------------------------------------------------------------
  Map store_map(const OutStore& st) {
    const Node& n = g.nodes[st.node];
    Map m;
    if (st.level == 3) {
      m.co.assign(n.rank(), idx_const(d.nd(), 0));
      return m;
    }
    if (st.level == 2 || st.level == 1) {
      // row level: the row digits; column level: the FIN kernel's digits
      int k = 0;
      for (int64_t s : n.shape) m.co.push_back(s == 1 ? idx_const(d.nd(), 0) : idx_digit(d.nd(), k++));
      return m;
    }
    // element level
    if (elem) {
      m.lin = true;
      m.l = idx_const(d.nd(), 0);
      for (int j = 0; j < d.nd(); ++j) m.l.c[j] = d.iw[j];
      return m;
    }
    // same non-unit extents as the seed reduction's operand
    const RedDef& seed = K.reds.front();
    const Node& x = g.nodes[g.nodes[seed.node].args[0]];
    std::vector<Idx> nu;
    for (size_t j = 0; j < x.shape.size(); ++j)
      if (x.shape[j] != 1) nu.push_back(seed.opmap.co[j]);
    size_t t = 0;
    for (int64_t s : n.shape) m.co.push_back(s == 1 ? idx_const(d.nd(), 0) : nu[t++]);
    return m;
  }

  std::string store_stmt_elem(const OutStore& st, int phase, const std::string& v) {
    const Node& n = g.nodes[st.node];
    Map m = store_map(st);
    Idx A = to_linear(m, n.shape, d);
    std::string ptr = ptr_of(st.node, true, st.port, st.temp_offset);
    std::string base;
    if (contiguous(A, &base)) {
      auto un = unrounded.find(v);
      if (n.dt == FGT_BF16 && K.vec % 2 == 0 && un != unrounded.end() && un->second.second.k == SC_LANE &&
          un->second.second.p == phase) {
        // the unrounded f32 values go out in pairs, rounded by the packed conversion
        std::string ob = fresh("obf");
        chunkpre[phase].push_back("float " + ob + "[" + std::to_string(K.vec) + "];");
        chunkpost[phase].push_back("fgt_vstore_bf16_rn(" + ptr + " + " + base + " + e0, " + ob + ");");
        return ob + "[v] = " + un->second.first + ";";
      }
      std::string ob = fresh("ob");
      chunkpre[phase].push_back(st_t(n.dt) + " " + ob + "[" + std::to_string(K.vec) + "];");
      chunkpost[phase].push_back("fgt_vstore(" + ptr + " + " + base + " + e0, " + ob + ");");
      return ob + "[v] = " + st_conv(n.dt, v) + ";";
    }
    return ptr + "[" + itext(A) + "] = " + st_conv(n.dt, v) + ";";
  }

  // Butterfly within TW lanes then (if the group spans warps) a combine of
  // the warp partials, so every lane ends with the same deterministic value.
  // The warp partials are combined either sequentially in warp order, or
  // (butterfly, NW a power of two) by every warp reading partial lane % NW and
  // running an xor butterfly over NW lanes: each node of that tree combines
  // the same two operands on every lane, only commuted, so all lanes of all
  // warps agree bit for bit. trailing_sync=false drops the barrier that
  // protects the partials from the next write; callers do that only when
  // another barrier always lies between this read and that write.
  void group_reduce(std::vector<std::string>& out, const std::vector<std::pair<RedText, std::string>>& accs,
                    int TW, bool cross_warp, int NW, const std::string& tag, bool butterfly = false,
                    bool trailing_sync = true, bool parity = false) {
    // parity: two partial buffers used on alternate rows (it_ & 1), so the
    // next row writes the other buffer and no trailing barrier is needed.
    const std::string PB = parity ? "[it_ & 1]" : "";
    const std::string PD = parity ? "[2]" : "";
    if (accs.empty()) return;
    // f32 max / min over a whole warp: one redux.sync instead of the butterfly
    auto redux = [&](const RedText& t) {
      return TW == 32 && !t.arg && t.acc_t == "float" && (t.op == FGT_OP_REDUCE_MAX || t.op == FGT_OP_REDUCE_MIN);
    };
    bool any_shfl = false;
    for (auto& [t, a] : accs) {
      if (redux(t)) out.push_back(a + " = fgt_redux_" + std::string(t.op == FGT_OP_REDUCE_MAX ? "max" : "min") + "(" + a + ");");
      else any_shfl = true;
    }
    if (any_shfl) out.push_back("#pragma unroll");
    if (any_shfl) out.push_back("for (int m_ = 1; m_ < " + std::to_string(TW) + "; m_ <<= 1) {");
    for (auto& [t, a] : accs) {
      if (redux(t)) continue;
      if (t.arg) {
        out.push_back("  { const " + t.acc_t + " ov = fgt_shfl_xor(" + a + ", m_); const fgt_i64 oi = fgt_shfl_xor(" + a +
                      "i, m_); " + arg_stmt(t, a, a + "i", "ov", "oi") + " }");
      } else {
        out.push_back("  { const " + t.acc_t + " ov = fgt_shfl_xor(" + a + ", m_); " + comb_stmt(t, a, "ov") + " }");
      }
    }
    if (any_shfl) out.push_back("}");
    if (!cross_warp) return;
    for (auto& [t, a] : accs) {
      kdecl.push_back("__shared__ __align__(16) " + t.acc_t + " sm_" + a + tag + PD + "[" + std::to_string(NW) + "];");
      if (t.arg) kdecl.push_back("__shared__ fgt_i64 smi_" + a + tag + PD + "[" + std::to_string(NW) + "];");
    }
    out.push_back("if ((tid & 31) == 0) {");
    for (auto& [t, a] : accs) {
      out.push_back("  sm_" + a + tag + PB + "[tid >> 5] = " + a + ";");
      if (t.arg) out.push_back("  smi_" + a + tag + PB + "[tid >> 5] = " + a + "i;");
    }
    out.push_back("}");
    out.push_back("__syncthreads();");
    if (butterfly && NW > 1 && (NW & (NW - 1)) == 0 && NW <= 32) {
      const std::string mask = std::to_string(NW - 1);
      bool any_arg = false;
      for (auto& [t, a] : accs) {
        if (!t.arg && P.opt.xw_tree) {
          // Every thread reads the NW warp partials (broadcast loads) and
          // folds them in the pairwise tree the butterfly forms, which is
          // the same value bit for bit, without its dependent shuffles.
          const std::string sm = "sm_" + a + tag + PB;
          std::vector<std::string> lv;
          for (int w = 0; w < NW; ++w) lv.push_back(sm + "[" + std::to_string(w) + "]");
          // f32 sums take two nodes of a level per FADD2 (the same two
          // operands per node, each rounded once)
          const bool pair2 = P.opt.lane_pairs && t.acc_t == "float" && t.op == FGT_OP_REDUCE_SUM && !t.storage;
          for (int lvl = 0; lv.size() > 1; ++lvl) {
            std::vector<std::string> nx;
            size_t i = 0;
            for (; pair2 && i + 3 < lv.size(); i += 4) {
              const std::string ta = a + tag + "_t" + std::to_string(lvl) + "_" + std::to_string(i / 2),
                                tb = a + tag + "_t" + std::to_string(lvl) + "_" + std::to_string(i / 2 + 1);
              out.push_back("const float2 " + ta + "_p2 = __fadd2_rn(make_float2(" + lv[i] + ", " + lv[i + 2] + "), make_float2(" +
                            lv[i + 1] + ", " + lv[i + 3] + ")); const float " + ta + " = " + ta + "_p2.x; const float " + tb +
                            " = " + ta + "_p2.y;");
              nx.push_back(ta);
              nx.push_back(tb);
            }
            for (; i + 1 < lv.size(); i += 2) {
              const std::string tv = a + tag + "_t" + std::to_string(lvl) + "_" + std::to_string(i / 2);
              out.push_back(t.acc_t + " " + tv + " = " + lv[i] + "; " + comb_stmt(t, tv, lv[i + 1]));
              nx.push_back(tv);
            }
            lv = nx;
          }
          out.push_back(a + " = " + lv[0] + ";");
        } else {
          any_arg = true;  // folded by the butterfly below
          out.push_back(a + " = sm_" + a + tag + PB + "[tid & " + mask + "];");
          if (t.arg) out.push_back(a + "i = smi_" + a + tag + PB + "[tid & " + mask + "];");
        }
      }
      if (any_arg) {
        out.push_back("#pragma unroll");
        out.push_back("for (int m_ = 1; m_ < " + std::to_string(NW) + "; m_ <<= 1) {");
        for (auto& [t, a] : accs) {
          if (!t.arg && P.opt.xw_tree) continue;
          if (!t.arg) {
            out.push_back("  { const " + t.acc_t + " ov = fgt_shfl_xor(" + a + ", m_); " + comb_stmt(t, a, "ov") + " }");
            continue;
          }
          out.push_back("  { const " + t.acc_t + " ov = fgt_shfl_xor(" + a + ", m_); const fgt_i64 oi = fgt_shfl_xor(" + a +
                        "i, m_); " + arg_stmt(t, a, a + "i", "ov", "oi") + " }");
        }
        out.push_back("}");
      }
      cluster_exchange(out, accs, tag);
      if (trailing_sync) out.push_back("__syncthreads();");
      return;
    }
    for (auto& [t, a] : accs) {
      out.push_back(a + " = sm_" + a + tag + "[0];");
      if (t.arg) out.push_back(a + "i = smi_" + a + tag + "[0];");
      out.push_back("for (int w_ = 1; w_ < " + std::to_string(NW) + "; ++w_) {");
      if (t.arg)
        out.push_back("  { const " + t.acc_t + " ov = sm_" + a + tag + "[w_]; const fgt_i64 oi = smi_" + a + tag + "[w_]; " +
                      arg_stmt(t, a, a + "i", "ov", "oi") + " }");
      else out.push_back("  { const " + t.acc_t + " ov = sm_" + a + tag + "[w_]; " + comb_stmt(t, a, "ov") + " }");
      out.push_back("}");
    }
    out.push_back("__syncthreads();");
  }

  // Row split over a cluster: every CTA holds its part of each reduction (the
  // same value in all its threads); thread 0 publishes it in a two-deep ring
  // (cx_ counts exchanges), one cluster barrier makes the parts visible, and
  // every thread combines them in rank order, so all CTAs agree bit for bit.
  // The next exchange's barrier orders these reads before the ring slot is
  // written again.
  void cluster_exchange(std::vector<std::string>& out, const std::vector<std::pair<RedText, std::string>>& accs,
                        const std::string& tag) {
    if (K.cluster <= 1) return;
    const std::string CL = std::to_string(K.cluster);
    auto xt = [](const std::string& t) { return t == "bool" ? std::string("int") : t; };
    for (auto& [t, a] : accs) {
      kdecl.push_back("__shared__ " + xt(t.acc_t) + " smc_" + a + tag + "[2];");
      if (t.arg) kdecl.push_back("__shared__ fgt_i64 smci_" + a + tag + "[2];");
    }
    out.push_back("if (tid == 0) {");
    for (auto& [t, a] : accs) {
      out.push_back("  smc_" + a + tag + "[cx_ & 1] = (" + xt(t.acc_t) + ")" + a + ";");
      if (t.arg) out.push_back("  smci_" + a + tag + "[cx_ & 1] = " + a + "i;");
    }
    out.push_back("}");
    out.push_back("fgt_cluster_sync();");
    for (auto& [t, a] : accs) {
      out.push_back(a + " = (" + t.acc_t + ")fgt_dsmem_ld(&smc_" + a + tag + "[cx_ & 1], 0u);");
      if (t.arg) out.push_back(a + "i = fgt_dsmem_ld(&smci_" + a + tag + "[cx_ & 1], 0u);");
      out.push_back("for (unsigned q_ = 1; q_ < " + CL + "u; ++q_) {");
      if (t.arg)
        out.push_back("  { const " + t.acc_t + " ov = (" + t.acc_t + ")fgt_dsmem_ld(&smc_" + a + tag + "[cx_ & 1], q_); " +
                      "const fgt_i64 oi = fgt_dsmem_ld(&smci_" + a + tag + "[cx_ & 1], q_); " + arg_stmt(t, a, a + "i", "ov", "oi") +
                      " }");
      else
        out.push_back("  { const " + t.acc_t + " ov = (" + t.acc_t + ")fgt_dsmem_ld(&smc_" + a + tag + "[cx_ & 1], q_); " +
                      comb_stmt(t, a, "ov") + " }");
      out.push_back("}");
    }
    out.push_back("++cx_;");
  }

  std::string arg_index(const RedDef& rd) {
    const Node& n = g.nodes[rd.node];
    const Node& x = g.nodes[n.args[0]];
    auto C = to_coords(rd.opmap, x.shape, d);
    std::string t = itext(C[n.attrs[0]]);
    return t;
  }

  // ------------------------------------------------------------ kernels --
  std::string args_struct() {
    const int nin = std::max<int>(1, (int)g.input_nodes.size());
    const int nout = std::max<int>(1, (int)g.outputs.size());
    // kernels exchanging records through the peer mailboxes also get every
    // rank's mailbox, the communicator's status word, this rank and the wait limit
    const std::string x = K.fin_stage == 3 ? " unsigned char* xmb[" + std::to_string(kXMaxWorld) +
                                                 "]; unsigned* xstat; long long xrank; unsigned long long xlimit;"
                                           : "";
    return "struct FgtArgs { const void* in[" + std::to_string(nin) + "]; void* out[" + std::to_string(nout) +
           "]; unsigned char* ws; long long nparts; long long pad_;" + x + " };\n";
  }

  static void put(std::ostringstream& o, const std::vector<std::string>& v, const std::string& ind) {
    for (auto& s : v)
      if (!s.empty()) o << ind << s << "\n";
  }

  std::string digits_o() {
    std::string s;
    for (int k = 0; k < d.no(); ++k)
      s += "const fgt_i64 o" + std::to_string(k) + " = (r / " + std::to_string(d.ow[k]) + "LL) % " + std::to_string(d.od[k]) + "LL; ";
    return s;
  }
  // Element digits. When the innermost extent is a whole number of vector
  // chunks, every element of the chunk at e0 shares its outer digits and the
  // innermost one is e0's plus the lane offset `vv`; the digits are then taken
  // from e0 (unsigned: e0 >= 0), which the unrolled lanes share.
  bool chunk_digits() const {
    return !d.id.empty() && d.iw.back() == 1 && K.vec > 1 && d.id.back() % K.vec == 0;
  }
  std::string digits_i(bool from_e0 = false, const std::string& vv = "v") {
    std::string s;
    const int n = (int)d.id.size();
    // digits below 2^30 are 32-bit values: the guards and offsets built on
    // them then compare and add in 32 bits where the compiler can narrow them
    bool narrow = true;
    for (int64_t m : d.id) narrow = narrow && m < (int64_t(1) << 30);
    for (int k = 0; k < n; ++k) {
      const std::string w = std::to_string(d.iw[k]), m = std::to_string(d.id[k]);
      if (from_e0 && chunk_digits())
        s += std::string(narrow ? "const int i" : "const fgt_i64 i") + std::to_string(k) + " = (" +
             (narrow ? "int" : "fgt_i64") + ")(((unsigned long long)e0 / " + w + "ULL) % " + m + "ULL)" +
             (k == n - 1 ? " + " + vv : std::string()) + "; ";
      else
        s += "const fgt_i64 i" + std::to_string(k) + " = (e / " + w + "LL) % " + m + "LL; ";
    }
    return s;
  }

  std::string build_row() {
    // every chunk of the row is in range when the (nonempty) row is a whole
    // number of thread-chunks; the bound check is then left out
    // (with column tiles: a whole number of tiles)
    const int64_t span = K.col_tiles > 1 ? K.tile_elems : (int64_t)K.tpr * K.vec;
    const std::string CHK = d.NI > 0 && d.NI % span == 0 ? "if (true)" : "if (e0 < NI)";
    // Phases: one element loop per dependency level of the row reductions.
    std::vector<const RedDef*> rows, cols;
    for (auto& rd : K.reds) (rd.role == ROLE_ROW ? rows : cols).push_back(&rd);
    int maxp = 0;
    std::map<int, int> rphase;
    for (auto* rd : rows) {
      an.run(rd->node, [&] {
        Map m;
        const Node& n = g.nodes[rd->node];
        int k = 0;
        for (int64_t s : n.shape) m.co.push_back(s == 1 ? idx_const(d.nd(), 0) : idx_digit(d.nd(), k++));
        return m;
      }());
      rphase[rd->node] = an.red_phase[rd->node];
      maxp = std::max(maxp, rphase[rd->node]);
    }
    std::map<const RedDef*, int> cphase;
    for (auto* rd : cols) {
      int p = an.run(g.nodes[rd->node].args[0], rd->opmap).phase;
      cphase[rd] = p;
      maxp = std::max(maxp, p);
    }
    std::vector<std::pair<const OutStore*, int>> estores;
    for (auto& st : K.stores)
      if (st.level == 0) {
        int p = an.run(st.node, store_map(st)).phase;
        estores.push_back({&st, p});
        maxp = std::max(maxp, p);
      }
    nphase = maxp + 1;
    rowsc.assign(nphase + 1, {});
    lane.assign(nphase, {});
    chunkpre.assign(nphase, {});
    chunkpost.assign(nphase, {});
    post.assign(nphase, {});
    const int TW = std::min(K.tpr, 32);
    const bool xw = K.tpr > 32;
    const int NW = K.nt / 32;
    // row reductions
    std::map<int, std::vector<std::pair<RedText, std::string>>> phase_accs;
    std::map<int, std::string> acc_of;
    for (auto* rd : rows) {
      RedText t = red_text(g, rd->node, P.opt.accumulation, CTX_ROW);
      int p = rphase[rd->node];
      std::string a = fresh("acc");
      rowsc[p].push_back(t.acc_t + " " + a + " = " + t.ident + ";");
      if (t.arg) rowsc[p].push_back("fgt_i64 " + a + "i = " + t.identi + ";");
      std::string v = val(g.nodes[rd->node].args[0], rd->opmap, Sc{SC_LANE, p});
      // Value reductions over a register-resident row run four independent
      // accumulator chains (element k of the thread's row pieces feeds chain
      // k % 4), folded pairwise before the group combine: four dependent
      // chains instead of one. Storage-dtype accumulation keeps one chain.
      const bool chains = !t.arg && !t.storage && !K.streaming && K.nch * K.vec >= 4;
      // max/min of a widened bf16 register row: packed bf16x2 max/min over
      // the row's 32-bit words (exact: no rounding), folded into the f32
      // accumulator after the phase.
      std::string pk_site;  // the chunk's words of the site (text valid in the chunk loop)
      {
        auto te = texpr.find(v);
        const std::string& ex = te == texpr.end() ? v : te->second;
        const bool pk = pack16(FGT_BF16);
        const std::string pre = pk ? "fgt_bf16_to_f32(fgt_h16(" : "fgt_bf16_to_f32(", suf = pk ? "[c], v))" : "[c][v])";
        const std::string lsuf = pk ? ", v))" : "[v])";  // a ring-resident phase-local array
        const bool maxmin = (t.op == FGT_OP_REDUCE_MAX || t.op == FGT_OP_REDUCE_MIN) && t.fl && !t.storage && cached &&
                            K.vec % 2 == 0 && ex.compare(0, pre.size(), pre) == 0;
        if (maxmin && ex.size() > pre.size() + suf.size() && ex.compare(ex.size() - suf.size(), suf.size(), suf) == 0) {
          const std::string site = ex.substr(pre.size(), ex.size() - pre.size() - suf.size());
          for (auto& rs : row_sites)
            if (rs.name == site && rs.st == (pk ? "fgt_u32" : "fgt_u16") && !rs.uniform) pk_site = site + "[c]";
        }
        if (maxmin && pk_site.empty() && ex.size() > pre.size() + lsuf.size() &&
            ex.compare(ex.size() - lsuf.size(), lsuf.size(), lsuf) == 0) {
          const std::string loc = ex.substr(pre.size(), ex.size() - pre.size() - lsuf.size());
          auto rl = resident_loc.find(loc);
          if (rl != resident_loc.end() && row_sites[rl->second].st == (pk ? "fgt_u32" : "fgt_u16")) pk_site = loc;
        }
      }
      resets[p].push_back(a + " = " + t.ident + ";");
      if (!pk_site.empty()) {
        const bool mx = t.op == FGT_OP_REDUCE_MAX;
        const std::string init = mx ? "0xff80ff80u" : "0x7f807f80u";
        rowsc[p].push_back("fgt_u32 " + a + "_pk = " + init + ";");
        resets[p].push_back(a + "_pk = " + init + ";");
        chunkpost[p].push_back(a + "_pk = fgt_" + (mx ? std::string("max") : std::string("min")) + "_bf16x2_row(" + a + "_pk, " +
                               pk_site + ");");
        post[p].push_back(comb_stmt(t, a, "fgt_bf16_to_f32((fgt_u16)(" + a + "_pk & 0xffffu))"));
        post[p].push_back(comb_stmt(t, a, "fgt_bf16_to_f32((fgt_u16)(" + a + "_pk >> 16))"));
        phase_accs[p].push_back({t, a});
        acc_of[rd->node] = a;
        red_var[rd->node] = fresh("red");
        continue;
      }
      if (t.arg) resets[p].push_back(a + "i = " + t.identi + ";");
      if (chains)
        for (int k = 0; k < 4; ++k) resets[p].push_back(a + "_s[" + std::to_string(k) + "] = " + t.ident + ";");
      if (t.arg) {
        lane[p].push_back("{ const fgt_i64 ix = " + arg_index(*rd) + "; " + scan_stmt(t, a, a + "i", v, "ix") + " }");
      } else if (chains) {
        rowsc[p].push_back(t.acc_t + " " + a + "_s[4] = {" + t.ident + ", " + t.ident + ", " + t.ident + ", " + t.ident +
                           "};");
        lane[p].push_back(comb_stmt(t, a + "_s[(c * " + std::to_string(K.vec) + " + v) & 3]", v));
        if (t.acc_t == "float" && t.op == FGT_OP_REDUCE_SUM && !t.storage) f32_sum_accs.insert(a + "_s");
        post[p].push_back(comb_stmt(t, a + "_s[0]", a + "_s[1]"));
        post[p].push_back(comb_stmt(t, a + "_s[2]", a + "_s[3]"));
        post[p].push_back(comb_stmt(t, a + "_s[0]", a + "_s[2]"));
        post[p].push_back(comb_stmt(t, a, a + "_s[0]"));
      } else {
        lane[p].push_back(comb_stmt(t, a, v));
      }
      phase_accs[p].push_back({t, a});
      acc_of[rd->node] = a;
      std::string rv = fresh("red");
      red_var[rd->node] = rv;
    }
    // With two or more cross-warp phases per row, the barrier of the next
    // phase separates each phase's partial reads from its next row's writes.
    // A single cross-warp phase alternates two partial buffers by row instead.
    const bool single = phase_accs.size() == 1 && xw && (NW & (NW - 1)) == 0;
    parity_rows = single;
    row_phases = (int)phase_accs.size();
    for (auto& [p, accs] : phase_accs) {
      group_reduce(post[p], accs, TW, xw, NW, "_p" + std::to_string(p), true, false, single);
    }
    for (auto* rd : rows) {
      int p = rphase[rd->node];
      RedText t = red_text(g, rd->node, P.opt.accumulation, CTX_ROW);
      const std::string& a = acc_of[rd->node];
      if (t.arg) {
        std::string ix = a + "i";
        if (rd->index_offset) ix = "(" + ix + "+" + std::to_string(rd->index_offset) + "LL)";
        post[p].push_back("const fgt_i64 " + red_var[rd->node] + " = " + ix + ";");
      } else {
        post[p].push_back("const " + vt_t(t.dt) + " " + red_var[rd->node] + " = " + finalize(t, a, t.acc_t) + ";");
      }
    }
    // column reductions: per-thread accumulators across the CTA's rows, in
    // registers, or (FGT_ROW_SMEM_COLS) in a thread-private shared-memory
    // region at the start of the dynamic shared memory: slot
    // ((c * VEC/4 + v/4) * NT + tid) * 4 + v%4 keeps a thread's four
    // consecutive elements in one 16-byte word and neighbouring threads'
    // words adjacent (no bank conflicts for 16-byte accesses)
    std::vector<std::string> colfin, colfin_pre;
    // or (FGT_ROW_TMEM_COLS) in tensor memory: f32 sums of a one-row-per-CTA
    // kernel of a multiple of 128 threads whose rows are whole numbers of
    // thread chunks (every tcgen05 access is warp-wide). Thread t of warp w
    // owns TMEM lane 32 * (w % 4) + t and the columns
    // (w / 4) * n * NCH * VEC + k * NCH * VEC + c * VEC + v (accumulator k of n,
    // chunk c, element v); a phase loads chunk c's accumulators, updates
    // them and stores them back.
    auto tmem_ok = [&](const RedText& t) {
      return P.opt.tmem_cols && cached && K.cluster == 1 && K.col_tiles <= 1 && K.tpr == K.nt && K.nt % 128 == 0 &&
             (K.vec == 4 || K.vec == 8 || K.vec == 16) && d.NI > 0 && d.NI % ((int64_t)K.tpr * K.vec) == 0 && !t.arg &&
             t.acc_t == "float";
    };
    int n_tm = 0;
    for (auto* rd : cols)
      if (tmem_ok(red_text(g, rd->node, P.opt.accumulation, CTX_COL))) ++n_tm;
    const int64_t tm_pt = (int64_t)K.nch * K.vec;
    const bool use_tm = n_tm > 0 && (int64_t)(K.nt / 128) * n_tm * tm_pt <= 512;
    if (use_tm) {
      tm_alloc = 32;
      while (tm_alloc < (int64_t)(K.nt / 128) * n_tm * tm_pt) tm_alloc *= 2;
      kdecl.push_back("__shared__ unsigned tm_slot_;");
      kdecl.push_back("if ((tid >> 5) == 0) fgt_tm_alloc(&tm_slot_, " + std::to_string(tm_alloc) + "u);");
      kdecl.push_back("fgt_tm_fence_before(); __syncthreads(); fgt_tm_fence_after();");
      kdecl.push_back("const unsigned tm_thr_ = tm_slot_ + ((unsigned)(((tid >> 5) & 3) * 32) << 16) + (unsigned)((tid >> 7) * " +
                      std::to_string(n_tm * tm_pt) + ");");
    }
    int k_tm = 0;
    for (auto* rd : cols) {
      RedText t = red_text(g, rd->node, P.opt.accumulation, CTX_COL);
      int p = cphase[rd];
      col_phases.insert(p);
      std::string a = fresh("cacc");
      const bool in_tmem = use_tm && tmem_ok(t);
      const bool in_smem = !in_tmem && P.opt.smem_cols && K.cluster == 1 && !t.arg;
      std::string el = a + "[c][v]";
      if (in_tmem) {
        const std::string tma = "tm_" + a, ta = "ta_" + a, VS = std::to_string(K.vec), NS = std::to_string(K.nch);
        el = ta + "[v]";
        kdecl.push_back("const unsigned " + tma + " = tm_thr_ + " + std::to_string(k_tm * tm_pt) + "u;");
        kdecl.push_back("{ float z_[" + VS + "]; for (int v = 0; v < " + VS + "; ++v) z_[v] = " + t.ident + "; for (int c = 0; c < " +
                        NS + "; ++c) fgt_tm_st(" + tma + " + c * " + VS + ", z_); }");
        const std::string ld = "float " + ta + "[" + VS + "]; fgt_tm_ld(" + ta + ", " + tma + " + c * " + VS + ");";
        chunkpre[p].push_back(ld);
        chunkpost[p].push_back("fgt_tm_st(" + tma + " + c * " + VS + ", " + ta + ");");
        colfin_pre.push_back(ld);
        tm_phases.insert(p);
        ++k_tm;
      } else if (in_smem) {
        const int64_t esz = t.acc_t == "double" ? 8 : 4;
        const std::string NTC = std::to_string(K.nt);
        if (K.vec % 4 == 0)
          el = a + "[((c * " + std::to_string(K.vec / 4) + " + v / 4) * " + NTC + " + tid) * 4 + v % 4]";
        else
          el = a + "[(c * " + std::to_string(K.vec) + " + v) * " + NTC + " + tid]";
        kdecl.push_back(t.acc_t + "* const " + a + " = (" + t.acc_t + "*)(fgt_dsmem + " + std::to_string(col_smem) + ");");
        col_smem += ((int64_t)K.nt * K.nch * K.vec * esz + 15) / 16 * 16;
      } else {
        std::string dims = "[" + std::to_string(K.nch) + "][" + std::to_string(K.vec) + "]";
        kdecl.push_back(t.acc_t + " " + a + dims + ";");
        if (t.arg) kdecl.push_back("fgt_i64 " + a + "i" + dims + ";");
      }
      if (!in_tmem) {
        std::string init = "for (int c = 0; c < " + std::to_string(K.nch) + "; ++c) for (int v = 0; v < " + std::to_string(K.vec) +
                           "; ++v) { " + el + " = " + t.ident + ";" + (t.arg ? " " + a + "i[c][v] = " + t.identi + ";" : std::string()) +
                           " }";
        kdecl.push_back(init);
      }
      std::string v = val(g.nodes[rd->node].args[0], rd->opmap, Sc{SC_LANE, p});
      if (t.arg) {
        std::string ix = arg_index(*rd);
        if (rd->index_offset) ix = "(" + ix + "+" + std::to_string(rd->index_offset) + "LL)";
        lane[p].push_back("{ const fgt_i64 ix = " + ix + "; " + scan_stmt(t, a + "[c][v]", a + "i[c][v]", v, "ix") + " }");
      } else {
        lane[p].push_back(comb_stmt(t, el, v));
        if (t.acc_t == "float" && t.op == FGT_OP_REDUCE_SUM && !t.storage) f32_sum_accs.insert(in_tmem ? "ta_" + a : a);
      }
      std::string slot = "(" + std::string(K.cluster > 1 ? "(fgt_i64)(blockIdx.x / " + std::to_string(K.cluster) + ")"
                                                          : "(fgt_i64)blockIdx.x") +
                         " * " + std::to_string(K.rows_per_cta) + " + grp)";
      std::string pv = "((" + t.part_t + "*)(p.ws+" + std::to_string(rd->part_val) + "LL))";
      std::string body = pv + "[" + slot + "*" + std::to_string(d.NI) + "LL + e] = (" + t.part_t + ")" + el + ";";
      if (t.arg) body += " ((fgt_i64*)(p.ws+" + std::to_string(rd->part_idx) + "LL))[" + slot + "*" + std::to_string(d.NI) +
                         "LL + e] = " + a + "i[c][v];";
      colfin.push_back(body);
    }
    if (use_tm) kdecl.push_back("fgt_tm_wait_st();");
    // element stores
    for (auto& [st, p] : estores) {
      std::string v = val(st->node, store_map(*st), Sc{SC_LANE, p});
      lane[p].push_back(store_stmt_elem(*st, p, v));
    }
    // row-level stores (after the last phase)
    for (auto& st : K.stores) {
      if (st.level != 1) continue;
      Map m = store_map(st);
      std::string v = val(st.node, m, Sc{SC_ROW, nphase});
      const Node& n = g.nodes[st.node];
      Idx A = to_linear(m, n.shape, d);
      rowend.push_back("if (rv && lane == 0) " + ptr_of(st.node, true, st.port, st.temp_offset) + "[" + itext(A) + "] = " +
                       st_conv(n.dt, v) + ";");
    }
    // ---- assemble
    std::ostringstream o;
    const std::string NT = std::to_string(K.nt), TPR = std::to_string(K.tpr), VEC = std::to_string(K.vec),
                      NCH = std::to_string(K.nch), RPC = std::to_string(K.rows_per_cta);
    // element offset of chunk c of this thread; column tiles add the tile's base
    const std::string E0 = (K.col_tiles > 1 ? "(fgt_i64)blockIdx.y * " + std::to_string(K.tile_elems) + "LL + " : std::string()) +
                           "((fgt_i64)c * " + TPR + " + lane) * " + VEC;
    o << args_struct();
    if (K.cluster > 1) {
      // one row over a cluster: the row's thread index spans the cluster's CTAs
      o << "extern \"C\" __global__ void __cluster_dims__(" << K.cluster << ", 1, 1) __launch_bounds__(" << NT << ") " << K.name
        << "(const FgtArgs p) {\n  fgt_pdl_enter();\n";
      o << "  const int tid = threadIdx.x; const unsigned crank = fgt_cluster_rank(); const int lane = (int)crank * " << NT
        << " + tid; const int grp = 0;\n";
    } else {
      o << "extern \"C\" __global__ void __launch_bounds__(" << NT << ") " << K.name << "(const FgtArgs p) {\n  fgt_pdl_enter();\n";
      o << "  const int tid = threadIdx.x; const int lane = tid % " << TPR << "; const int grp = tid / " << TPR << ";\n";
    }
    o << "  (void)lane; (void)grp;\n";
    o << "  extern __shared__ __align__(16) unsigned char fgt_dsmem[];\n";
    o << "  const fgt_i64 NR = " << d.NR << "LL, NI = " << d.NI << "LL; (void)NI;\n";
    put(o, kdecl, "  ");
    if (cached && !prolane.empty()) {
      o << "  #pragma unroll\n  for (int c = 0; c < " << NCH << "; ++c) {\n";
      o << "    const fgt_i64 e0 = " << E0 << ";\n";
      o << "    " << CHK << " {\n";
      put(o, prosites, "      ");
      o << "      #pragma unroll\n      for (int v = 0; v < " << VEC << "; ++v) {\n";
      o << "        const fgt_i64 e = e0 + v; " << digits_i(true) << "\n";
      put(o, prolane, "        ");
      o << "      }\n    }\n  }\n";
    }
    // ---- streamed row operands: the current row is in registers, the next
    // row is in flight while the current one is computed:
    // (a) staged operands travel global -> shared memory with cp.async (no
    //     registers held by data in flight) and are copied to registers when
    //     the row starts; every thread copies and reads only its own pieces;
    // (b) other operands are double-buffered in registers.
    std::vector<RowSite*> staged_sites, reg_sites;
    for (auto& rs : row_sites) (rs.staged ? staged_sites : reg_sites).push_back(&rs);
    const bool res = resident() && !staged_sites.empty();
    if (!staged_sites.empty()) {
      // rows in flight per CTA: as many as fit the ring budget (96 KB: two CTAs per SM);
      // ring-resident rows keep the current row in a stage too (at least two)
      stages = (int)std::min<int64_t>(8, std::max<int64_t>(res ? 2 : 1, ((int64_t)P.opt.ring_kb * 1024) / std::max<int64_t>(1, stage_bytes)));
      int64_t off = col_smem;  // the ring follows any shared-memory column accumulators
      for (auto* rs : staged_sites) {
        rs->smem_off = off;
        off += (int64_t)stages * K.rows_per_cta * K.nch * (K.tpr / K.cluster) * rs->bytes;
      }
    }
    if (res) {
      // phase-local copies read the current row's stage `stg`
      for (auto& cp : chunkpre)
        for (auto& st : cp)
          for (size_t k = 0; k < row_sites.size(); ++k) {
            const std::string ph = "@PIECE" + std::to_string(k) + "@";
            for (size_t at = st.find(ph); at != std::string::npos; at = st.find(ph))
              st.replace(at, ph.size(), piece_off(row_sites[k], "stg"));
          }
    }
    const std::string stride = K.cluster > 1 ? "(fgt_i64)(gridDim.x / " + std::to_string(K.cluster) + ") * " + RPC
                                             : "(fgt_i64)gridDim.x * " + RPC;
    const std::string CB = K.cluster > 1 ? "(fgt_i64)(blockIdx.x / " + std::to_string(K.cluster) + ")" : "(fgt_i64)blockIdx.x";
    auto chunk_loop = [&](std::ostringstream& os, const std::string& ind, const std::function<void(const std::string&)>& body) {
      os << ind << "#pragma unroll\n" << ind << "for (int c = 0; c < " << NCH << "; ++c) {\n";
      os << ind << "  const fgt_i64 e0 = " << E0 << ";\n";
      os << ind << "  " << CHK << " {\n";
      body(ind + "    ");
      os << ind << "  }\n" << ind << "}\n";
    };
    auto reg_loads = [&](std::ostringstream& os, const std::string& ind, const char* rvar, bool next) {
      chunk_loop(os, ind, [&](const std::string& in) {
        for (auto* rs : reg_sites) os << in << site_load(*rs, next ? rs->name + "_n" : rs->name, rvar) << "\n";
      });
    };
    auto issue = [&](std::ostringstream& os, const std::string& ind, const char* rvar, const std::string& stg) {
      chunk_loop(os, ind, [&](const std::string& in) {
        for (auto* rs : staged_sites)
          os << in << "fgt_cp_async<" << rs->bytes << ">(sbase_ + " << piece_off(*rs, stg) << ", " << rs->ptr << " + "
             << itext(rs->addr, "e", rvar) << " + e0);\n";
      });
    };
    auto smem_to_regs = [&](std::ostringstream& os, const std::string& ind, const std::string& stg) {
      chunk_loop(os, ind, [&](const std::string& in) {
        for (auto* rs : staged_sites)
          os << in << "fgt_lds(" << rs->name << "[c], (const " << rs->st << "*)(fgt_dsmem + " << piece_off(*rs, stg) << "));\n";
      });
    };
    for (auto& rs : row_sites) {
      if (res && rs.staged) continue;  // read from the ring by each phase
      const std::string W = rs.packed ? std::to_string(K.vec / 2) : VEC;
      std::string dims = rs.uniform ? "[" + NCH + "]" : "[" + NCH + "][" + W + "]";
      o << "  " << rs.st << " " << rs.name << dims << ";";
      if (!rs.staged) o << " " << rs.st << " " << rs.name << "_n" << dims << ";";
      o << "\n";
    }
    if (stages) o << "  const unsigned sbase_ = fgt_smem_addr(fgt_dsmem);\n";
    // Ring invariant at the top of iteration i: registers hold row i, ring
    // stage (i+k) % S holds row i+k for k = 1..S (S cp.async groups pending).
    // Ring-resident rows: stage i % S holds row i and stages of rows i+1 ..
    // i+S-1 are in flight; the wait at the top of the iteration completes
    // row i's group, and its stage refills with row i+S once the row is done.
    const std::string S = std::to_string(stages);
    if (!row_sites.empty()) {
      o << "  { const fgt_i64 r0_ = " << CB << " * " << RPC << " + grp;\n    if (r0_ < NR) {\n";
      reg_loads(o, "      ", "r0_", false);
      o << "    }\n";
      if (res) {
        o << "    for (int k_ = 0; k_ < " << S << "; ++k_) {\n";
        o << "      const fgt_i64 rk_ = r0_ + (fgt_i64)k_ * " << stride << ";\n      if (rk_ < NR) {\n";
        issue(o, "        ", "rk_", "k_");
        o << "      }\n      fgt_cp_commit();\n    }\n";
      } else if (stages) {
        o << "    for (int k_ = 0; k_ < " << S << "; ++k_) {\n";
        o << "      const fgt_i64 rk_ = r0_ + (fgt_i64)k_ * " << stride << ";\n      if (rk_ < NR) {\n";
        issue(o, "        ", "rk_", "k_");
        o << "      }\n      fgt_cp_commit();\n    }\n";
        o << "    fgt_cp_wait<" << stages - 1 << ">();\n";
        smem_to_regs(o, "    ", "0");
        o << "    { const fgt_i64 rk_ = r0_ + (fgt_i64)" << S << " * " << stride << ";\n      if (rk_ < NR) {\n";
        issue(o, "        ", "rk_", "0");
        o << "      }\n      fgt_cp_commit();\n    }\n";
      }
      o << "  }\n";
      if (res) o << "  int stg = 0;\n";
      else if (stages) o << "  int stg = " << (stages > 1 ? 1 : 0) << ";\n";
    }
    if (!rowpf_first.empty()) {
      o << "  { const fgt_i64 r = " << CB << " * " << RPC << " + grp; const bool rv = r < NR; " << digits_o() << "\n";
      put(o, rowpf_first, "    ");
      o << "  }\n";
    }
    if (parity_rows) o << "  int it_ = 0;\n";
    if (K.cluster > 1 && xw) o << "  int cx_ = 0;\n";
    o << "  for (fgt_i64 rb = " << CB << " * " << RPC << "; rb < NR; rb += " << stride << ") {\n";
    o << "    const fgt_i64 r = rb + grp; const bool rv = r < NR; " << digits_o() << "\n";
    if (!rowpf.empty()) {
      put(o, rowpf, "    ");
      o << "    { const fgt_i64 rpf_ = r + " << stride << ";\n";
      o << "      { const fgt_i64 r = rpf_; const bool rv = r < NR; " << digits_o() << "\n";
      put(o, rowpf_next, "        ");
      o << "      }\n    }\n";
    }
    if (!reg_sites.empty()) {
      o << "    const fgt_i64 rn_ = r + " << stride << ";\n    if (rn_ < NR) {\n";
      reg_loads(o, "      ", "rn_", true);
      o << "    }\n";
    }
    if (res) o << "    fgt_cp_wait<" << stages - 1 << ">();\n";
    put(o, rowdecl, "    ");
    auto phase_loop = [&](int p, const std::vector<std::string>& body, const std::string& ind) {
      if (cached) o << ind << "  #pragma unroll\n";
      else o << ind << "  #pragma unroll 1\n";
      o << ind << "  for (int c = 0; c < " << NCH << "; ++c) {\n";
      o << ind << "    const fgt_i64 e0 = " << E0 << ";\n";
      o << ind << "    " << CHK << " {\n";
      put(o, chunkpre[p], ind + "      ");
      o << ind << "      #pragma unroll\n";
      if (pairs()) {
        o << ind << "      " << pair_header(VEC);
        put(o, pair_body(body), ind + "        ");
      } else {
        o << ind << "      for (int v = 0; v < " << VEC << "; ++v) {\n";
        o << ind << "        const fgt_i64 e = e0 + v; " << digits_i(true) << "\n";
        put(o, body, ind + "        ");
      }
      o << ind << "      }\n";
      put(o, chunkpost[p], ind + "      ");
      o << ind << "    }\n" << ind << "  }\n";
    };
    for (int p = 0; p < nphase; ++p) {
      put(o, rowsc[p], "    ");
      // Divisions of a phase without column updates are checked once per
      // thread and phase: trackers of min/max |q| (NaN propagates into the
      // max); a thread whose quotients left the exact range resets its row
      // accumulators and redoes the phase with IEEE division. Redoing is
      // safe: the phase's other effects (cached values, element stores) are
      // overwritten with the same values.
      // Exps of such a phase by fgt_exp_q note max |x| the same way, and the
      // redo computes them with expf.
      const bool track = (div_phases.count(p) || exp_phases.count(p)) && !col_phases.count(p) && cached;
      const std::string dx = "dgx" + std::to_string(p), dn = "dgn" + std::to_string(p), de = "dge" + std::to_string(p);
      // Narrow division (FGT_ROW_NARROW_DIV, partitions whose floating outputs
      // are all 16-bit): x * RN(1/d) with no range notes; the phase is redone
      // with IEEE division only when a row's divisor has no normal reciprocal
      // (fgt_recip_for_div's NaN).
      const bool narrow = narrow_div();
      std::string rcp_ok;
      if (narrow && div_rcps.count(p))
        for (auto& rc : div_rcps[p]) rcp_ok += " && fgt_rcp_ok(" + rc + ")";
      if (track)
        o << "    float " << dx << " = 0.0f, " << dn << " = __int_as_float(0x7f800000), " << de << " = 0.0f;\n";
      if (p > 0 && P.opt.phase_copies && cached) {
        // the phase reads its operands through opaque copies (fgt_opaque): the
        // compiler then cannot merge its element values with the earlier
        // phases' and keep them live across the barriers in between
        for (auto& rs : row_sites) {
          if (res && rs.staged) continue;
          if (rs.uniform) o << "    for (int c = 0; c < " << NCH << "; ++c) fgt_opaque(" << rs.name << "[c]);\n";
          else
            o << "    for (int c = 0; c < " << NCH << "; ++c) for (int k = 0; k < " << (rs.packed ? K.vec / 2 : K.vec)
              << "; ++k) fgt_opaque(" << rs.name << "[c][k]);\n";
        }
        for (auto& [nm, w] : persisted_arrays)
          o << "    for (int c = 0; c < " << NCH << "; ++c) for (int k = 0; k < " << w << "; ++k) fgt_opaque(" << nm << "[c][k]);\n";
      }
      // this phase's TMEM loads follow the earlier rows' stores of the same columns
      if (tm_phases.count(p)) o << "    fgt_tm_wait_st();\n";
      o << "    if (rv) {\n";
      phase_loop(p,
                 track ? div_form(lane[p], narrow ? "@MUL@" : "fgt_div_q",
                                  narrow ? "" : "fgt_div_note(" + dx + ", " + dn + ", ", "fgt_exp_q", "fgt_exp_note(" + de + ", ")
                       : div_form(lane[p], narrow ? "fgt_div_nby" : "fgt_div_by", ""),
                 "    ");
      o << "    }\n";
      if (track) {
        o << "    if (rv && !(fgt_div_ok(" << dx << ", " << dn << ") && fgt_exp_ok(" << de << ")" << rcp_ok << ")) {\n";
        put(o, resets[p], "      ");
        phase_loop(p, div_form(lane[p], "fgt_div_ieee", ""), "    ");
        o << "    }\n";
      }
      put(o, post[p], "    ");
    }
    put(o, rowsc[nphase], "    ");
    put(o, rowend, "    ");
    for (auto* rs : reg_sites) {
      if (rs->uniform) o << "    for (int c = 0; c < " << NCH << "; ++c) " << rs->name << "[c] = " << rs->name << "_n[c];\n";
      else o << "    for (int c = 0; c < " << NCH << "; ++c) for (int v = 0; v < " << (rs->packed ? std::to_string(K.vec / 2) : VEC) << "; ++v) " << rs->name << "[c][v] = " << rs->name << "_n[c][v];\n";
    }
    if (res) {
      // row i is done: its stage refills with row i+S
      o << "    { const fgt_i64 rk_ = r + (fgt_i64)" << S << " * " << stride << ";\n      if (rk_ < NR) {\n";
      issue(o, "        ", "rk_", "stg");
      o << "      }\n      fgt_cp_commit();\n    }\n";
      o << "    stg = stg + 1 == " << S << " ? 0 : stg + 1;\n";
    } else if (stages) {
      // row i+1 -> registers; its stage refills with row i+1+S
      o << "    fgt_cp_wait<" << stages - 1 << ">();\n";
      smem_to_regs(o, "    ", "stg");
      o << "    { const fgt_i64 rk_ = r + (fgt_i64)" << stages + 1 << " * " << stride << ";\n      if (rk_ < NR) {\n";
      issue(o, "        ", "rk_", "stg");
      o << "      }\n      fgt_cp_commit();\n    }\n";
      o << "    stg = stg + 1 == " << S << " ? 0 : stg + 1;\n";
    }
    if (parity_rows) o << "    ++it_;\n";
    o << "  }\n";
    if (stages) o << "  fgt_cp_wait<0>();\n";
    // no CTA of a cluster leaves while a peer may still read its shared
    // memory (the last exchange has no later barrier of its own)
    if (K.cluster > 1) o << "  fgt_cluster_sync();\n";
    if (!colfin.empty()) {
      if (use_tm) o << "  fgt_tm_wait_st();\n";
      o << "  #pragma unroll\n  for (int c = 0; c < " << NCH << "; ++c) {\n";
      o << "    const fgt_i64 e0 = " << E0 << ";\n";
      o << "    " << CHK << " {\n";
      put(o, colfin_pre, "      ");
      o << "      #pragma unroll\n      for (int v = 0; v < " << VEC << "; ++v) {\n";
      o << "        const fgt_i64 e = e0 + v;\n";
      put(o, colfin, "        ");
      o << "      }\n    }\n  }\n";
    }
    if (use_tm) {
      // every warp is done with tensor memory before warp 0 frees it
      o << "  fgt_tm_fence_before();\n  __syncthreads();\n  fgt_tm_fence_after();\n";
      o << "  if ((tid >> 5) == 0) fgt_tm_dealloc(tm_slot_, " << tm_alloc << "u);\n";
    }
    o << "}\n";
    return o.str();
  }

  // scatter_add accumulator type and pointer text
  std::string scatter_acc_t() const {
    const Node& n = g.nodes[K.scatter_node];
    if (is_float(n.dt)) return "double";
    return n.dt == FGT_I64 ? "unsigned long long" : "int";
  }
  std::string scatter_acc_ptr() const {
    return "((" + scatter_acc_t() + "*)(p.ws+" + std::to_string(K.scatter_acc) + "LL))";
  }
  // Bucket lists of a row scatter: head[r] is the last update scattered to
  // base row r (-1: none) and next[i] the update after update i in its row's
  // list (ints; RA = R rounded up to 4 keeps next 16-byte aligned).
  std::string ll_head() const { return "((int*)(p.ws+" + std::to_string(K.scatter_acc) + "LL))"; }
  std::string ll_next() const {
    const int64_t RA = (g.nodes[K.scatter_node].shape[0] + 3) / 4 * 4;
    return "((int*)(p.ws+" + std::to_string(K.scatter_acc + 4 * RA) + "LL))";
  }
  // bucket sums: f64 for floats (rounded once with the base), unsigned
  // (wrapping) for integers
  std::string csr_acc_t() const {
    const Node& n = g.nodes[K.scatter_node];
    if (is_float(n.dt)) return "double";
    return n.dt == FGT_I64 ? "unsigned long long" : "unsigned int";
  }
  std::string build_elem() {
    nphase = 1;
    rowsc.assign(2, {});
    lane.assign(1, {});
    chunkpre.assign(1, {});
    chunkpost.assign(1, {});
    post.assign(1, {});
    std::vector<std::pair<RedText, std::string>> accs;
    std::vector<std::string> partial_store;
    if (K.scatter_stage == 1) lane[0].push_back(scatter_acc_ptr() + "[e] = 0;");
    if (K.scatter_stage == 11) lane[0].push_back(ll_head() + "[e] = -1;");
    if (K.scatter_stage == 12) {
      // over the indices: each in-range index's update becomes the head of its
      // row's list, the previous head its next (order within a list free)
      const Node& n = g.nodes[K.scatter_node];
      Map mi;
      mi.lin = true;
      mi.l = idx_const(d.nd(), 0);
      for (int j = 0; j < d.nd(); ++j) mi.l.c[j] = d.iw[j];
      const std::string iv = val(n.args[1], mi, Sc{SC_LANE, 0});
      const std::string R = std::to_string(n.shape[0]) + "LL";
      const std::string body = ll_next() + "[e] = atomicExch(" + ll_head() + " + gi_, (int)e);";
      lane[0].push_back("{ const fgt_i64 gi_ = (fgt_i64)(" + iv + "); if (gi_ >= 0LL && gi_ < " + R + ") " + body + " }");
    }
    if (K.scatter_stage == 2) {
      // updates domain: base offset of update i = its coordinates with the
      // scattered axis replaced by indices[i]
      const Node& n = g.nodes[K.scatter_node];
      const Node& base = g.nodes[n.args[0]];
      const Node& up = g.nodes[n.args[2]];
      const int ax = (int)n.attrs[0], ir = g.nodes[n.args[1]].rank();
      Map mu;
      mu.lin = true;
      mu.l = idx_const(d.nd(), 0);
      for (int j = 0; j < d.nd(); ++j) mu.l.c[j] = d.iw[j];
      auto C = to_coords(mu, up.shape, d);
      Map mi;
      for (int k = 0; k < ir; ++k) mi.co.push_back(C[ax + k]);
      const std::string uv = val(n.args[2], mu, Sc{SC_LANE, 0});
      const std::string iv = val(n.args[1], mi, Sc{SC_LANE, 0});
      auto bst = row_major_strides(base.shape);
      std::string off = "gi_*" + std::to_string(bst[ax]) + "LL";
      for (int k = 0; k < ax; ++k) off += "+" + itext(C[k]) + "*" + std::to_string(bst[k]) + "LL";
      for (int k = ax + 1; k < base.rank(); ++k) off += "+" + itext(C[k - 1 + ir]) + "*" + std::to_string(bst[k]) + "LL";
      const std::string A = scatter_acc_t();
      lane[0].push_back("{ const fgt_i64 gi_ = (fgt_i64)(" + iv + "); if (gi_ >= 0LL && gi_ < " + std::to_string(base.shape[ax]) +
                        "LL) atomicAdd(" + scatter_acc_ptr() + " + (" + off + "), (" + A + ")(" + uv + ")); }");
    }
    for (auto& rd : K.reds) {
      RedText t = red_text(g, rd.node, P.opt.accumulation, CTX_FULL);
      std::string a = fresh("acc");
      kdecl.push_back(t.acc_t + " " + a + " = " + t.ident + ";");
      if (t.arg) kdecl.push_back("fgt_i64 " + a + "i = " + t.identi + ";");
      std::string v = val(g.nodes[rd.node].args[0], rd.opmap, Sc{SC_LANE, 0});
      // Two-level accumulation: the VEC lanes of a chunk reduce with a 32-bit
      // lane index, then the chunk folds into the thread accumulator (64-bit
      // indices) once per chunk. Sums and products keep the accumulator's type
      // in the lanes too (f64 for f32), so a whole-tensor sum rounds once.
      const std::string la = a + "l";
      const std::string lt = t.acc_t;
      const std::string lident = t.ident;
      const std::string ix = arg_index(rd);
      if (t.arg && ix == "(0LL+1LL*e)") {
        chunkpre[0].push_back(lt + " " + la + " = " + t.ident + "; int " + la + "i = 0x7fffffff;");
        lane[0].push_back(scan_stmt(t, la, la + "i", v, "v"));
        std::string gi = "e0 + " + la + "i";
        if (rd.index_offset) gi += " + " + std::to_string(rd.index_offset) + "LL";
        chunkpost[0].push_back("{ const fgt_i64 gi = " + gi + "; " + scan_stmt(t, a, a + "i", la, "gi") + " }");
      } else if (t.arg) {
        std::string gx = ix;
        if (rd.index_offset) gx = "(" + gx + "+" + std::to_string(rd.index_offset) + "LL)";
        lane[0].push_back("{ const fgt_i64 ix = " + gx + "; " + scan_stmt(t, a, a + "i", v, "ix") + " }");
      } else {
        chunkpre[0].push_back(lt + " " + la + " = " + lident + ";");
        lane[0].push_back(comb_stmt(t, la, v));
        chunkpost[0].push_back(comb_stmt(t, a, la));
      }
      accs.push_back({t, a});
      std::string ps = "((" + t.part_t + "*)(p.ws+" + std::to_string(rd.part_val) + "LL))[blockIdx.x] = (" + t.part_t + ")" + a + ";";
      if (t.arg) ps += " ((fgt_i64*)(p.ws+" + std::to_string(rd.part_idx) + "LL))[blockIdx.x] = " + a + "i;";
      partial_store.push_back(ps);
    }
    for (auto& st : K.stores) {
      std::string v = val(st.node, store_map(st), Sc{SC_LANE, 0});
      lane[0].push_back(store_stmt_elem(st, 0, v));
    }
    std::vector<std::string> red_code;
    group_reduce(red_code, accs, 32, true, K.nt / 32, "_f");
    std::ostringstream o;
    const std::string NT = std::to_string(K.nt), VEC = std::to_string(K.vec), UU = std::to_string(U);
    o << args_struct();
    // the row-scatter bucket sums wait on dependent loads (list head, next link,
    // update row): more resident warps hide more of that latency
    const std::string LB = K.scatter_csr && K.scatter_stage == 3 ? NT + ", 8" : NT;
    o << "extern \"C\" __global__ void __launch_bounds__(" << LB << ") " << K.name << "(const FgtArgs p) {\n  fgt_pdl_enter();\n";
    o << "  const int tid = threadIdx.x; const fgt_i64 r = 0; const bool rv = true; (void)r; (void)rv;\n";
    o << "  const fgt_i64 NI = " << d.NI << "LL; const fgt_i64 NCK = NI / " << VEC << ";\n";
    put(o, kdecl, "  ");
    o << "  const fgt_i64 stride = (fgt_i64)gridDim.x * " << NT << ";\n";
    o << "  for (fgt_i64 base = (fgt_i64)blockIdx.x * " << NT << " + tid; base < NCK; base += stride * " << UU << ") {\n";
    put(o, rowdecl, "    ");
    if (!eload.empty()) {
      o << "    #pragma unroll\n    for (int u = 0; u < " << UU << "; ++u) {\n";
      o << "      const fgt_i64 ch = base + u * stride;\n      if (ch < NCK) {\n        const fgt_i64 e0 = ch * " << VEC << ";\n";
      put(o, eload, "        ");
      o << "      }\n    }\n";
    }
    o << "    #pragma unroll\n    for (int u = 0; u < " << UU << "; ++u) {\n";
    o << "      const fgt_i64 ch = base + u * stride;\n      if (ch < NCK) {\n        const fgt_i64 e0 = ch * " << VEC << ";\n";
    put(o, chunkpre[0], "        ");
    o << "        #pragma unroll\n";
    if (pairs()) {
      o << "        " << pair_header(VEC);
      put(o, pair_body(lane[0]), "          ");
    } else {
      o << "        for (int v = 0; v < " << VEC << "; ++v) {\n";
      o << "          const fgt_i64 e = e0 + v; " << digits_i(true) << "\n";
      put(o, lane[0], "          ");
    }
    o << "        }\n";
    put(o, chunkpost[0], "        ");
    o << "      }\n    }\n  }\n";
    if (!accs.empty()) {
      put(o, red_code, "  ");
      o << "  if (tid == 0) {\n";
      put(o, partial_store, "    ");
      o << "  }\n";
    }
    o << "}\n";
    return o.str();
  }

  // Combine partials for reduction rd into `a` (+ `a`i), per element e.
  std::string fin_combine(const RedDef& rd, const RedText& t, const std::string& src_t, const std::string& a,
                          const std::string& e, const std::string& count, int stage, int64_t rec_off, bool xchg = false) {
    std::ostringstream s;
    const std::string M = std::to_string(rd.M);
    if (stage == 2) {
      // ranks' records: gathered by NCCL into the workspace, or (xchg) delivered
      // by the ranks into this rank's mailbox, read past L1 (written by peers)
      std::string recb = xchg ? "(p.xmb[p.xrank]+" + std::to_string(kXDataOff) + "LL+(fgt_i64)(xe_ & 1u)*" +
                                    std::to_string(kXMaxWorld * kXSlot) + "LL)"
                              : "(p.ws+" + std::to_string(K.recv_offset) + "LL)";
      const std::string stride = std::to_string(xchg ? kXSlot : K.record_bytes);
      std::string pv = "((const " + t.part_t + "*)(" + recb + "+(fgt_i64)w_*" + stride + "LL+" + std::to_string(rec_off) + "LL))";
      std::string pi = "((const fgt_i64*)(" + recb + "+(fgt_i64)w_*" + stride + "LL+" + std::to_string(rec_off + rd.M * 8) +
                       "LL))";
      const std::string ld0 = "", ld1 = "";
      std::string lo = rd.combine_ranks ? "0" : (xchg ? "(int)p.xrank" : std::to_string(P.opt.rank));
      std::string hi = rd.combine_ranks ? std::to_string(P.opt.world) : (xchg ? "(int)p.xrank + 1" : std::to_string(P.opt.rank + 1));
      s << "for (int w_ = " << lo << "; w_ < " << hi << "; ++w_) { ";
      if (xchg) {
        // this rank's mailbox slot of rank w_: the record words are requested
        // for every rank first (llpre, emitted before the combines), then each
        // is taken, or waited for when it does not carry this launch's epoch yet
        const std::string slot = recb + "+(fgt_i64)w_*" + stride + "LL";
        const std::string W = std::to_string(P.opt.world);
        const std::string off = std::to_string(rec_off) + "LL + (fgt_i64)(" + e + ") * 8LL";
        const std::string offi = std::to_string(rec_off + rd.M * 8) + "LL + (fgt_i64)(" + e + ") * 8LL";
        const std::string lw = "llw_" + a;
        const bool wide = t.part_t == "double" || t.part_t == "fgt_i64" || t.part_t == "fgt_u64";
        std::string pre = "fgt_u64 " + lw + "[" + W + "][4]; " + "\n#pragma unroll\nfor (int w_ = " + lo + "; w_ < " + hi +
                          "; ++w_) { " + lw + "[w_ - (" + lo + ")][0] = fgt_ll_raw(" + slot + ", " + off + "); " + lw +
                          "[w_ - (" + lo + ")][1] = " + (wide ? "fgt_ll_raw(" + slot + ", " + off + " + 4)" : std::string("0")) + ";";
        if (t.arg)
          pre += " " + lw + "[w_ - (" + lo + ")][2] = fgt_ll_raw(" + slot + ", " + offi + "); " + lw + "[w_ - (" + lo +
                 ")][3] = fgt_ll_raw(" + slot + ", " + offi + " + 4);";
        pre += " }";
        llpre.push_back(pre);
        const std::string vv = "fgt_ll_value<" + t.part_t + ">(" + lw + "[w_ - (" + lo + ")][0], " + lw + "[w_ - (" + lo +
                               ")][1], " + slot + ", " + off + ", xe_, t0_, p.xlimit, p.xstat)";
        if (t.arg)
          s << "{ const " << t.part_t << " ov = " << vv << "; const fgt_i64 oi = fgt_ll_value<fgt_i64>(" << lw << "[w_ - (" << lo
            << ")][2], " << lw << "[w_ - (" << lo << ")][3], " << slot << ", " << offi << ", xe_, t0_, p.xlimit, p.xstat); "
            << arg_stmt(t, a, a + "i", "ov", "oi") << " }";
        else s << "{ const " << t.fin_t << " ov = (" << t.fin_t << ")" << vv << "; " << comb_stmt(t, a, "ov") << " }";
        s << " }";
        return s.str();
      }
      if (t.arg) s << "{ const " << t.part_t << " ov = " << ld0 << pv << "[" << e << "]" << ld1 << "; const fgt_i64 oi = " << ld0
                   << pi << "[" << e << "]" << ld1 << "; " << arg_stmt(t, a, a + "i", "ov", "oi") << " }";
      else s << "{ const " << t.fin_t << " ov = (" << t.fin_t << ")" << ld0 << pv << "[" << e << "]" << ld1 << "; "
             << comb_stmt(t, a, "ov") << " }";
      s << " }";
      return s.str();
    }
    std::string pv = "((const " + src_t + "*)(p.ws+" + std::to_string(rd.part_val) + "LL))";
    std::string pi = "((const fgt_i64*)(p.ws+" + std::to_string(rd.part_idx) + "LL))";
    // FULLFIN: the CTA's threads stride over the partials; COLFIN: each of
    // the kColGroups warps of a CTA sums every kColGroups-th partial of its
    // 32 columns (pg_ is the warp's group)
    const bool full = K.kind == KKind::FULLFIN;
    const std::string Q0 = full ? "tid" : "pg_", QS = full ? std::to_string(K.nt) : std::to_string(kColGroups);
    if (!t.arg && !full) {
      // four partials' loads in flight per step, combined in order (the same
      // sums as one partial at a time)
      s << "for (int once_ = 0; once_ < 1; ++once_) { fgt_i64 q_ = " << Q0 << "; for (; q_ + 3 * " << QS << " < " << count
        << "; q_ += 4 * " << QS << ") { ";
      for (int k = 0; k < 4; ++k)
        s << "const " << t.fin_t << " o" << k << "_ = (" << t.fin_t << ")" << pv << "[(q_ + " << k << " * " << QS << ")*" << M
          << "LL+" << e << "]; ";
      for (int k = 0; k < 4; ++k) s << comb_stmt(t, a, "o" + std::to_string(k) + "_") << " ";
      s << "} for (; q_ < " << count << "; q_ += " << QS << ") { const " << t.fin_t << " ov = (" << t.fin_t << ")" << pv << "[q_*"
        << M << "LL+" << e << "]; " << comb_stmt(t, a, "ov") << " } }";
      return s.str();
    }
    s << "for (fgt_i64 q_ = " << Q0 << "; q_ < " << count << "; q_ += " << QS << ") { ";
    if (t.arg) s << "{ const " << src_t << " ov = " << pv << "[q_*" << M << "LL+" << e << "]; const fgt_i64 oi = " << pi << "[q_*"
                 << M << "LL+" << e << "]; " << arg_stmt(t, a, a + "i", "ov", "oi") << " }";
    else s << "{ const " << t.fin_t << " ov = (" << t.fin_t << ")" << pv << "[q_*" << M << "LL+" << e << "]; " << comb_stmt(t, a, "ov") << " }";
    s << " }";
    return s.str();
  }

  // COLFIN layout: a CTA handles 32 consecutive columns with kColGroups warps,
  // warp g summing partials g, g + kColGroups, ...; the group sums are then
  // combined in group order (a fixed order: every launch gives the same bits).
  static constexpr int kColGroups = 8;

  // Column loop of a COLFIN kernel over blocks of 32 columns: the partial
  // sums of the CTA's warps, their combination in group order by warp 0, then
  // `tail` (per column e, warp 0 only).
  void col_partial_loop(std::ostringstream& o, const std::vector<std::string>& comb,
                        const std::vector<std::pair<RedText, std::string>>& accs, const std::vector<std::string>& tail) {
    const std::string G = std::to_string(kColGroups);
    o << "  const fgt_i64 NI = " << d.NI << "LL;\n";
    o << "  const int cl_ = tid & 31, pg_ = tid >> 5;\n";
    for (auto& [t, a] : accs) {
      o << "  __shared__ " << t.fin_t << " cg_" << a << "[" << G << "][32];\n";
      if (t.arg) o << "  __shared__ fgt_i64 cgi_" << a << "[" << G << "][32];\n";
    }
    o << "  for (fgt_i64 cb_ = blockIdx.x; cb_ * 32 < NI; cb_ += gridDim.x) {\n";
    o << "    const fgt_i64 e = cb_ * 32 + cl_;\n";
    o << "    const bool ev_ = e < NI;\n";
    // accumulator declarations, then the partial loops under the bound check
    std::vector<std::string> decls, loops;
    for (const std::string& st : comb) (st.compare(0, 4, "for ") == 0 ? loops : decls).push_back(st);
    put(o, decls, "    ");
    o << "    if (ev_) {\n";
    put(o, loops, "      ");
    o << "    }\n";
    for (auto& [t, a] : accs) {
      o << "    cg_" << a << "[pg_][cl_] = " << a << ";\n";
      if (t.arg) o << "    cgi_" << a << "[pg_][cl_] = " << a << "i;\n";
    }
    o << "    __syncthreads();\n";
    o << "    if (pg_ == 0 && ev_) {\n";
    o << "      " << digits_i() << "\n";
    for (auto& [t, a] : accs) {
      o << "      for (int g_ = 1; g_ < " << G << "; ++g_) { ";
      if (t.arg) o << "const " << t.fin_t << " ov = cg_" << a << "[g_][cl_]; const fgt_i64 oi = cgi_" << a << "[g_][cl_]; "
                   << arg_stmt(t, a, a + "i", "ov", "oi");
      else o << "const " << t.fin_t << " ov = cg_" << a << "[g_][cl_]; " << comb_stmt(t, a, "ov");
      o << " }\n";
    }
    put(o, tail, "      ");
    o << "    }\n    __syncthreads();\n  }\n";
  }

  std::string build_fin() {
    nphase = 1;
    rowsc.assign(2, {});
    lane.assign(1, {});
    chunkpre.assign(1, {});
    chunkpost.assign(1, {});
    post.assign(1, {});
    const bool col = K.kind == KKind::COLFIN;
    const int stage = K.fin_stage;
    const bool xchg = stage == 3;  // stages 1 and 2 with the records exchanged through the peer mailboxes
    std::vector<std::string> comb, rec_write, comb2;
    std::vector<std::pair<RedText, std::string>> accs;
    std::vector<std::string> finals;
    int64_t rec_off = 0;
    for (auto& rd : K.reds) {
      RedText t = red_text(g, rd.node, P.opt.accumulation, CTX_FIN);
      // partials are stored in the producer's partial type
      const std::string src_t = red_text(g, rd.node, P.opt.accumulation, col ? CTX_COL : CTX_FULL).part_t;
      std::string a = fresh("fa");
      comb.push_back(t.fin_t + " " + a + " = " + t.ident + ";");
      if (t.arg) comb.push_back("fgt_i64 " + a + "i = " + t.identi + ";");
      comb.push_back(fin_combine(rd, t, src_t, a, col ? "e" : "0", "p.nparts", xchg ? 1 : stage, rec_off));
      accs.push_back({t, a});
      if (xchg) {
        comb2.push_back(t.fin_t + " " + a + " = " + t.ident + ";");
        if (t.arg) comb2.push_back("fgt_i64 " + a + "i = " + t.identi + ";");
        comb2.push_back(fin_combine(rd, t, src_t, a, col ? "e" : "0", "p.nparts", 2, rec_off, true));
      }
      if (xchg) {
        // record words (value, epoch) into rank k_'s slot for this rank
        const std::string ei = col ? "e" : "0";
        rec_write.push_back("fgt_ll_put<" + t.part_t + ">(xrec_, " + std::to_string(rec_off) + "LL + (fgt_i64)(" + ei +
                            ") * 8LL, (" + t.part_t + ")" + a + ", xe_);");
        if (t.arg)
          rec_write.push_back("fgt_ll_put<fgt_i64>(xrec_, " + std::to_string(rec_off + rd.M * 8) + "LL + (fgt_i64)(" + ei +
                              ") * 8LL, " + a + "i, xe_);");
      } else if (stage == 1) {
        std::string recb = "(p.ws+" + std::to_string(K.send_offset) + "LL+" + std::to_string(rec_off) + "LL)";
        rec_write.push_back("((" + t.part_t + "*)" + recb + ")[" + (col ? "e" : "0") + "] = (" + t.part_t + ")" + a + ";");
        if (t.arg)
          rec_write.push_back("((fgt_i64*)(" + recb + "+" + std::to_string(rd.M * 8) + "LL))[" + (col ? "e" : "0") + "] = " + a + "i;");
      }
      rec_off += rd.M * 8 * (t.arg ? 2 : 1);
      std::string fv = fresh("fin");
      red_var[rd.node] = fv;
      if (t.arg) finals.push_back("const fgt_i64 " + fv + " = " + a + "i;");
      else finals.push_back("const " + vt_t(t.dt) + " " + fv + " = " + finalize(t, a, t.fin_t) + ";");
    }
    if (stage != 1) {
      for (auto& st : K.stores) {
        Map m = store_map(st);
        std::string v = val(st.node, m, Sc{SC_LANE, 0});
        const Node& n = g.nodes[st.node];
        Idx A = to_linear(m, n.shape, d);
        lane[0].push_back(ptr_of(st.node, true, st.port, st.temp_offset) + "[" + itext(A) + "] = " + st_conv(n.dt, v) + ";");
      }
    }
    // FULLFIN: one CTA; strided partial combine, then a block combine.
    std::vector<std::string> red_code;
    if (!col && stage != 2) group_reduce(red_code, accs, 32, true, K.nt / 32, "_fin");
    if (!col && stage != 2) {
      // one strided loop over the partials for all reductions (their loads in
      // flight together), unrolled; each accumulator still sees its partials
      // in the same order
      const std::string head = "for (fgt_i64 q_ = tid; q_ < p.nparts; q_ += " + std::to_string(K.nt) + ") { ";
      std::vector<std::string> decls;
      std::string bodies;
      bool ok = true;
      for (const std::string& st : comb) {
        if (st.compare(0, head.size(), head) == 0 && st.size() > head.size() + 2 && st.compare(st.size() - 2, 2, " }") == 0)
          bodies += st.substr(head.size(), st.size() - head.size() - 2) + " ";
        else if (st.compare(0, 4, "for ") == 0) ok = false;
        else decls.push_back(st);
      }
      if (ok && !bodies.empty()) {
        comb = decls;
        comb.push_back("#pragma unroll 4");
        comb.push_back(head + bodies + "}");
      }
    }
    std::ostringstream o;
    const std::string NT = std::to_string(K.nt);
    o << args_struct();
    o << "extern \"C\" __global__ void __launch_bounds__(" << NT << ") " << K.name << "(const FgtArgs p) {\n  fgt_pdl_enter();\n";
    o << "  const int tid = threadIdx.x; const fgt_i64 r = 0; const bool rv = true; (void)r; (void)rv;\n";
    put(o, kdecl, "  ");
    if (xchg) {
      // Exchange of this CTA's record through the peer mailboxes: the record is
      // stored as (value, epoch) words into every rank's data[epoch % 2][this
      // rank] (NVLink stores for peers); each rank then reads the words of all
      // ranks from its own mailbox, waiting for each to carry this launch's
      // epoch, bounded by p.xlimit ns from the start of the reads (a timeout
      // marks the communicator's status word and goes on). No fence or flag is
      // needed: a word's epoch and value arrive in one 64-bit store. A rank
      // writes a slot again only two launches later, after every rank has
      // finished the launch that read it (each launch reads every column of
      // every rank before it ends).
      const std::string W = std::to_string(P.opt.world), MW = std::to_string(kXMaxWorld);
      const std::string slot = "p.xmb[k_]+" + std::to_string(kXDataOff) + "LL+((fgt_i64)(xe_ & 1u)*" + MW +
                               "+p.xrank)*" + std::to_string(kXSlot) + "LL";
      // One epoch per launch, the same in every CTA (a word written by one CTA
      // index is read by others): every CTA reads the communicator's epoch
      // word, and the last CTA to have read it (counted in the word after it)
      // advances it for the next launch.
      const std::string EP = "((volatile unsigned*)(p.xmb[p.xrank]+" + std::to_string(kXEpochOff) + "LL))";
      o << "  __shared__ unsigned xep_;\n";
      o << "  if (tid == 0) {\n";
      o << "    xep_ = " << EP << "[0] + 1u;\n";
      o << "    __threadfence();\n";
      o << "    if (atomicAdd((unsigned*)" << EP << " + 1, 1u) == gridDim.x - 1) { " << EP << "[1] = 0u; " << EP
        << "[0] = xep_; }\n";
      o << "  }\n";
      o << "  __syncthreads();\n  const unsigned xe_ = xep_;\n";
      if (col) {
        std::vector<std::string> tail{"for (int k_ = 0; k_ < " + W + "; ++k_) {", "  unsigned char* const xrec_ = " + slot + ";"};
        for (auto& w : rec_write) tail.push_back("  " + w);
        tail.push_back("}");
        col_partial_loop(o, comb, accs, tail);
        // every column of every rank, one column per thread
        o << "  const unsigned long long t0_ = fgt_globaltimer();\n";
        o << "  for (fgt_i64 e = (fgt_i64)blockIdx.x * " << NT << " + tid; e < NI; e += (fgt_i64)gridDim.x * " << NT << ") {\n";
        o << "    " << digits_i() << "\n";
        put(o, llpre, "    ");
        put(o, comb2, "    ");
        put(o, finals, "    ");
        put(o, lane[0], "    ");
        o << "  }\n}\n";
        return o.str();
      }
      o << "  const fgt_i64 e = 0; (void)e;\n";
      put(o, comb, "  ");
      put(o, red_code, "  ");
      o << "  if (tid != 0) return;\n";
      o << "  for (int k_ = 0; k_ < " << W << "; ++k_) {\n";
      o << "    unsigned char* const xrec_ = " << slot << ";\n";
      put(o, rec_write, "    ");
      o << "  }\n";
      o << "  const unsigned long long t0_ = fgt_globaltimer();\n  {\n";
      put(o, llpre, "    ");
      put(o, comb2, "    ");
      put(o, finals, "    ");
      put(o, lane[0], "    ");
      o << "  }\n}\n";
      return o.str();
    }
    if (col && stage != 2) {
      std::vector<std::string> tail = rec_write;
      if (stage != 1) {
        tail = finals;
        tail.insert(tail.end(), lane[0].begin(), lane[0].end());
      }
      col_partial_loop(o, comb, accs, tail);
      o << "}\n";
      return o.str();
    }
    if (col) {
      // stage 2: this rank's combine of the ranks' gathered records, per column
      o << "  const fgt_i64 NI = " << d.NI << "LL;\n";
      o << "  for (fgt_i64 e = (fgt_i64)blockIdx.x * " << NT << " + tid; e < NI; e += (fgt_i64)gridDim.x * " << NT << ") {\n";
      o << "    " << digits_i() << "\n";
      put(o, comb, "    ");
      put(o, finals, "    ");
      put(o, lane[0], "    ");
      o << "  }\n}\n";
      return o.str();
    }
    o << "  const fgt_i64 e = 0; (void)e;\n";
    if (stage == 2) {
      o << "  if (tid != 0) return;\n";
      put(o, comb, "  ");
    } else {
      put(o, comb, "  ");
      put(o, red_code, "  ");
      o << "  if (tid != 0) return;\n";
    }
    if (stage == 1) {
      put(o, rec_write, "  ");
    } else {
      put(o, finals, "  ");
      put(o, lane[0], "  ");
    }
    o << "}\n";
    return o.str();
  }

  // Lane statements with the division placeholders resolved: @DIVQ@ becomes
  // `fn`, and the @NOTE@(q) statements become `note` + "q);" (dropped when
  // note is empty).
  static std::vector<std::string> div_form(const std::vector<std::string>& v, const std::string& fn,
                                           const std::string& note, const std::string& efn = "expf",
                                           const std::string& enote = "") {
    std::vector<std::string> out;
    for (const std::string& s0 : v) {
      std::string s = s0;
      if (s.compare(0, 7, "@NOTE@(") == 0) {
        if (!note.empty()) out.push_back(note + s.substr(7));
        continue;
      }
      if (s.compare(0, 8, "@ENOTE@(") == 0) {
        if (!enote.empty()) out.push_back(enote + s.substr(8));
        continue;
      }
      for (size_t at; (at = s.find("@DIVQ@")) != std::string::npos;) {
        if (fn != "@MUL@") {
          s.replace(at, 6, fn);
          continue;
        }
        // x * y with y = RN(1/d): the argument list (x, d, y) up to its closing parenthesis
        size_t e = at + 7;
        for (int depth = 1; e < s.size() && depth > 0; ++e) {
          if (s[e] == '(') ++depth;
          else if (s[e] == ')') --depth;
        }
        auto xa = split_args(s.substr(at + 7, e - 1 - (at + 7)));
        s.replace(at, e - at, "__fmul_rn(" + xa[0] + "," + xa[2] + ")");
      }
      for (size_t at; (at = s.find("@EXPQ@")) != std::string::npos;) s.replace(at, 6, efn);
      out.push_back(s);
    }
    return out;
  }

  // ---- lane pairs: element loops step v by 2 and run each statement for
  // lane v (slot a) and lane v + 1 (slot b). Slot b's statement is slot a's
  // with the names the body declares, the element index e and the index
  // digits i<k> renamed, and v read as (v + 1). f32 adds, multiplies, tracked
  // divisions by a row constant and pairable accumulations issue as one
  // f32x2 instruction for both slots (sm_100 FADD2 / FMUL2 / FFMA2: IEEE
  // round-to-nearest per lane, subnormals kept); every other statement runs
  // slot a, then slot b, so each accumulator sees its elements in order.
  struct Tok {
    std::string s;
    bool ident;
  };
  static std::vector<Tok> tokens(const std::string& x) {
    std::vector<Tok> out;
    size_t i = 0;
    while (i < x.size()) {
      const char ch = x[i];
      if (std::isalpha((unsigned char)ch) || ch == '_') {
        size_t j = i + 1;
        while (j < x.size() && (std::isalnum((unsigned char)x[j]) || x[j] == '_')) ++j;
        out.push_back({x.substr(i, j - i), true});
        i = j;
      } else if (std::isdigit((unsigned char)ch)) {
        size_t j = i + 1;
        while (j < x.size() && (std::isalnum((unsigned char)x[j]) || x[j] == '_' || x[j] == '.')) ++j;
        out.push_back({x.substr(i, j - i), false});
        i = j;
      } else {
        out.push_back({std::string(1, ch), false});
        ++i;
      }
    }
    return out;
  }
  // top-level comma split of a call's argument text
  static std::vector<std::string> split_args(const std::string& a) {
    std::vector<std::string> out;
    int depth = 0;
    size_t st = 0;
    for (size_t i = 0; i < a.size(); ++i) {
      const char ch = a[i];
      if (ch == '(' || ch == '[') ++depth;
      else if (ch == ')' || ch == ']') --depth;
      else if (ch == ',' && depth == 0) {
        out.push_back(a.substr(st, i - st));
        st = i + 1;
      }
    }
    out.push_back(a.substr(st));
    return out;
  }
  // `F(args)` -> args when x is exactly one call of F
  static bool call_of(const std::string& x, const std::string& f, std::string* args) {
    if (x.size() < f.size() + 2 || x.compare(0, f.size() + 1, f + "(") != 0 || x.back() != ')') return false;
    int depth = 0;
    for (size_t i = f.size(); i < x.size(); ++i) {
      if (x[i] == '(') ++depth;
      else if (x[i] == ')' && --depth == 0 && i + 1 != x.size()) return false;
    }
    *args = x.substr(f.size() + 1, x.size() - f.size() - 2);
    return true;
  }
  std::vector<std::string> pair_body(const std::vector<std::string>& body) const {
    std::set<std::string> renamed = {"e"};
    for (size_t k = 0; k < d.id.size(); ++k) renamed.insert("i" + std::to_string(k));
    for (const std::string& st : body) {
      auto T = tokens(st);
      for (size_t i = 1; i + 1 < T.size(); ++i) {
        if (!T[i].ident) continue;
        size_t n = i + 1;  // next non-space token: '=' but not '=='
        while (n < T.size() && T[n].s == " ") ++n;
        if (n >= T.size() || T[n].s != "=" || (n + 1 < T.size() && T[n + 1].s == "=")) continue;
        size_t j = i;  // previous non-space token
        while (j > 0 && T[j - 1].s == " ") --j;
        // a type before the name, or a comma (later declarators of one
        // declaration: the generated code has no other `, name =`)
        if (j > 0 && ((T[j - 1].ident && T[j - 1].s != "else" && T[j - 1].s != "return") || T[j - 1].s == ","))
          renamed.insert(T[i].s);
      }
    }
    auto slot_b = [&](const std::string& st) {
      std::string out;
      for (auto& t : tokens(st)) {
        if (t.ident && t.s == "v") out += "(v + 1)";
        else if (t.ident && renamed.count(t.s)) out += t.s + "_b";
        else out += t.s;
      }
      return out;
    };
    auto trim = [](std::string x) {
      while (!x.empty() && x.front() == ' ') x.erase(x.begin());
      while (!x.empty() && x.back() == ' ') x.pop_back();
      return x;
    };
    // negations N = (-X): an add of N pairs as a subtraction of X, written
    // fma(X, -1, A) (X * -1 is exact, so this is A - X rounded once)
    std::map<std::string, std::string> negs;
    for (const std::string& st : body) {
      const std::string a = trim(st);
      static const std::string cf = "const float ";
      const size_t eq = a.find(" = (-");
      if (a.compare(0, cf.size(), cf) != 0 || eq == std::string::npos || a.size() < eq + 7 ||
          a.compare(a.size() - 2, 2, ");") != 0)
        continue;
      const std::string n = a.substr(cf.size(), eq - cf.size()), x = a.substr(eq + 5, a.size() - eq - 7);
      auto T = tokens(x);
      if (T.size() == 1 && T[0].ident) negs[n] = x;
    }
    // "make_float2(A, B)" with the negated operands of both slots, when both are negations
    auto neg_pair = [&](const std::string& a, const std::string& b, std::string* out) {
      auto ia = negs.find(trim(a));
      if (ia == negs.end()) return false;
      *out = "make_float2(" + ia->second + ", " + slot_b(ia->second) + ")";
      return trim(b) == slot_b(trim(a));
    };
    std::vector<std::string> out;
    for (const std::string& sa : body) {
      const std::string sb = slot_b(sa);
      const std::string a = trim(sa), b = trim(sb);
      bool done = false;
      // const float N = [round](F(x,y)); / const float N = fgt_div_q(x,D,Y);
      static const std::string cf = "const float ";
      const size_t eq = a.find(" = ");
      if (a.compare(0, cf.size(), cf) == 0 && eq != std::string::npos && a.back() == ';' &&
          a.find(';') == a.size() - 1) {
        const std::string na = a.substr(cf.size(), eq - cf.size());
        const std::string nb = b.substr(cf.size(), b.find(" = ") - cf.size());
        std::string ea = a.substr(eq + 3, a.size() - eq - 4), eb = b.substr(b.find(" = ") + 3);
        eb.pop_back();
        std::string wrap, inner_a = ea, inner_b = eb, args;
        for (const char* w : {"fgt_rnd_bf16", "fgt_rnd_f16"}) {
          std::string ia, ib;
          if (call_of(ea, w, &ia) && call_of(eb, w, &ib)) {
            wrap = w;
            inner_a = ia;
            inner_b = ib;
          }
        }
        const std::string pv = na + "_p2";
        for (const char* f : {"__fadd_rn", "__fmul_rn"}) {
          std::string aa, ab;
          if (!call_of(inner_a, f, &aa) || !call_of(inner_b, f, &ab)) continue;
          auto xa = split_args(aa), xb = split_args(ab);
          if (xa.size() != 2 || xb.size() != 2) break;
          const bool add = std::string(f) == "__fadd_rn";
          auto rw = [&](const std::string& x) { return wrap.empty() ? x : wrap + "(" + x + ")"; };
          std::string expr, nx;
          if (add && neg_pair(xa[1], xb[1], &nx))
            expr = "__ffma2_rn(" + nx + ", make_float2(-1.0f, -1.0f), make_float2(" + xa[0] + ", " + xb[0] + "))";
          else if (add && neg_pair(xa[0], xb[0], &nx))
            expr = "__ffma2_rn(" + nx + ", make_float2(-1.0f, -1.0f), make_float2(" + xa[1] + ", " + xb[1] + "))";
          else
            expr = std::string(add ? "__fadd2_rn" : "__fmul2_rn") + "(make_float2(" + xa[0] + ", " + xb[0] +
                   "), make_float2(" + xa[1] + ", " + xb[1] + "))";
          out.push_back("const float2 " + pv + " = " + expr + "; const float " + na + " = " + rw(pv + ".x") +
                        "; const float " + nb + " = " + rw(pv + ".y") + ";");
          done = true;
          break;
        }
        std::string da, db;
        if (!done && wrap.empty() && call_of(ea, "fgt_exp_q", &da) && call_of(eb, "fgt_exp_q", &db) &&
            split_args(da).size() == 1) {
          out.push_back("const float2 " + pv + " = fgt_exp_q2(make_float2(" + da + ", " + db + ")); const float " + na + " = " +
                        pv + ".x; const float " + nb + " = " + pv + ".y;");
          done = true;
        }
        if (!done && wrap.empty() && call_of(ea, "fgt_div_q", &da) && call_of(eb, "fgt_div_q", &db)) {
          auto xa = split_args(da), xb = split_args(db);
          if (xa.size() == 3 && xb.size() == 3 && xa[1] == xb[1] && xa[2] == xb[2]) {
            out.push_back("const float2 " + pv + " = fgt_div_q2(make_float2(" + xa[0] + ", " + xb[0] + "), " + xa[1] + ", " +
                          xa[2] + "); const float " + na + " = " + pv + ".x; const float " + nb + " = " + pv + ".y;");
            done = true;
          }
        }
      }
      // L = L + X; over a registered f32 sum accumulator with distinct slots
      if (!done && eq != std::string::npos && a.back() == ';' && a.find(';') == a.size() - 1) {
        const std::string la = a.substr(0, eq), lb = b.substr(0, b.find(" = "));
        const std::string base = la.substr(0, la.find('['));
        const std::string ra = a.substr(eq + 3, a.size() - eq - 4);
        std::string rb = b.substr(b.find(" = ") + 3);
        rb.pop_back();
        if (f32_sum_accs.count(base) && la != lb && ra.compare(0, la.size() + 3, la + " + ") == 0 &&
            rb.compare(0, lb.size() + 3, lb + " + ") == 0) {
          const std::string xa = ra.substr(la.size() + 3), xb = rb.substr(lb.size() + 3);
          std::string nx;
          const std::string sum = neg_pair(xa, xb, &nx)
                                      ? "__ffma2_rn(" + nx + ", make_float2(-1.0f, -1.0f), make_float2(" + la + ", " + lb + "))"
                                      : "__fadd2_rn(make_float2(" + la + ", " + lb + "), make_float2(" + xa + ", " + xb + "))";
          out.push_back("{ const float2 s_ = " + sum + "; " + la + " = s_.x; " + lb + " = s_.y; }");
          done = true;
        }
      }
      // range notes of both slots in one three-input max / min (sm_100;
      // PTX ISA 8.8): the same value as two two-input steps, NaN included
      if (!done && P.opt.max3 && a.back() == ';') {
        std::string args;
        const std::string ca = a.substr(0, a.size() - 1);
        if (call_of(ca, "fgt_div_note", &args)) {
          auto x = split_args(args);
          if (x.size() == 3) {
            out.push_back("fgt_div_note2(" + x[0] + "," + x[1] + "," + x[2] + ", " + slot_b(trim(x[2])) + ");");
            done = true;
          }
        } else if (call_of(ca, "fgt_exp_note", &args)) {
          auto x = split_args(args);
          if (x.size() == 2) {
            out.push_back("fgt_exp_note2(" + x[0] + "," + x[1] + ", " + slot_b(trim(x[1])) + ");");
            done = true;
          }
        }
      }
      if (!done) {
        out.push_back(sa);
        out.push_back(sb);
      }
    }
    return out;
  }
  // loop header over lane pairs (slot b's element index and digits included)
  std::string pair_header(const std::string& vec) {
    std::string dg = digits_i(true), db;
    for (auto& t : tokens(digits_i(true, "(v + 1)")))
      db += (t.ident && (t.s == "e" || (t.s.size() > 1 && t.s[0] == 'i' && std::isdigit((unsigned char)t.s[1]))))
                ? t.s + "_b"
                : t.s;
    return "for (int v = 0; v < " + vec + "; v += 2) {\n" + "const fgt_i64 e = e0 + v; " + dg + "\n" +
           "const fgt_i64 e_b = e0 + v + 1; " + db + " (void)e_b;\n";
  }

  std::string build() {
    std::string src = row ? build_row() : elem ? build_elem() : build_fin();
    // kernels without per-phase tracking keep the per-element guarded division
    std::istringstream in(src);
    std::ostringstream out;
    for (std::string line; std::getline(in, line);) {
      const size_t k = line.find_first_not_of(' ');
      if (k != std::string::npos && (line.compare(k, 7, "@NOTE@(") == 0 || line.compare(k, 8, "@ENOTE@(") == 0)) continue;
      for (size_t at; (at = line.find("@DIVQ@")) != std::string::npos;) line.replace(at, 6, "fgt_div_by");
      for (size_t at; (at = line.find("@EXPQ@")) != std::string::npos;) line.replace(at, 6, "expf");
      out << line << "\n";
    }
    return out.str();
  }
};

}  // namespace

void generate_sources(Plan& plan) {
  // Later kernels first: a temp that no later kernel reads is not stored.
  std::set<int64_t> loaded;
  for (int i = (int)plan.kernels.size() - 1; i >= 0; --i) {
    KernelDef& k = plan.kernels[i];
    std::vector<OutStore> keep;
    for (auto& s : k.stores)
      if (s.port >= 0 || loaded.count(s.temp_offset)) keep.push_back(s);
    k.stores = keep;
    Emitter em(plan, k, &loaded);
    k.source = em.build();
    k.smem_bytes = em.col_smem + (int64_t)em.stages * em.stage_bytes;
    if (em.tm_alloc > 0) {
      // at most 512 / tm_alloc CTAs per SM may hold tensor memory at once: the
      // dynamic shared memory is padded so that no more are resident (a CTA
      // beyond them would wait in tcgen05.alloc for another to finish)
      const int64_t cap = 512 / em.tm_alloc;
      if (cap < 32) k.smem_bytes = std::max<int64_t>(k.smem_bytes, 233472 / (cap + 1));
    }
    k.row_phases = em.row_phases;
  }
}

}  // namespace fgt
