// fgt_plan.cpp — cutting a partition into fused kernels.
//
// Replaces ASK's partitioner (cpp/compiler.cpp:44-48, _ask/gpu.py:71). The
// reference materialises a reduction at a partition boundary whenever it is
// reused through a broadcast (docs/en/architecture/backend.md:68), so softmax
// costs >= 3 kernels there (tests/test_tensor_primitives.py:215-217). Here a
// reduction read back at its own row stays in registers: all reductions over
// the same row signature share one ROW kernel, with one phase per dependency
// level, and only reductions consumed at other index maps are materialised.
#include "fgt_plan.h"

#include <algorithm>
#include <cstdio>
#include <functional>
#include <sstream>

namespace fgt {

// ------------------------------------------------------------- Idx / Map ---
std::string Idx::key() const {
  std::ostringstream s;
  if (!aff) {
    s << "{" << code << "}";
    return s.str();
  }
  for (int64_t v : c) s << v << ",";
  s << "+" << k;
  return s.str();
}
std::string Map::key() const {
  std::string s = lin ? "L" + l.key() : "C";
  if (!lin)
    for (const Idx& i : co) s += "|" + i.key();
  if (!guard.empty()) s += "?" + guard;
  return s;
}

void Domain::finish() {
  NR = 1;
  NI = 1;
  ow.assign(od.size(), 1);
  iw.assign(id.size(), 1);
  for (int k = (int)od.size() - 1; k >= 0; --k) {
    ow[k] = NR;
    NR *= od[k];
  }
  for (int k = (int)id.size() - 1; k >= 0; --k) {
    iw[k] = NI;
    NI *= id[k];
  }
}

Idx idx_const(int nd, int64_t v) {
  Idx r;
  r.c.assign(nd, 0);
  r.k = v;
  return r;
}
Idx idx_digit(int nd, int k) {
  Idx r = idx_const(nd, 0);
  r.c[k] = 1;
  return r;
}

// Non-affine forms are carried as C text over digit variables o<k>/i<k> and
// the row/element linear indices r/e. They arise only from reshapes that
// split a digit; the generator never needs to reason about them.
static std::string idx_text(const Idx& a, const Domain& d) {
  if (!a.aff) return "(" + a.code + ")";
  std::ostringstream s;
  s << "(" << a.k << "LL";
  for (int k = 0; k < d.nd(); ++k) {
    if (!a.c[k]) continue;
    if (k < d.no()) s << "+" << a.c[k] << "LL*o" << k;
    else s << "+" << a.c[k] << "LL*i" << (k - d.no());
  }
  s << ")";
  return s.str();
}
bool idx_dep_o(const Idx& a, const Domain& d) {
  if (!a.aff) return a.dep_o;
  for (int k = 0; k < d.no(); ++k)
    if (a.c[k]) return true;
  return false;
}
bool idx_dep_i(const Idx& a, const Domain& d) {
  if (!a.aff) return a.dep_i;
  for (int k = d.no(); k < d.nd(); ++k)
    if (a.c[k]) return true;
  return false;
}
static Idx idx_opaque(const std::string& code, bool o, bool i) {
  Idx r;
  r.aff = false;
  r.code = code;
  r.dep_o = o;
  r.dep_i = i;
  return r;
}

// Linear index of a value of shape `shape` read at map m.
Idx to_linear(const Map& m, const Shape& shape, const Domain& d) {
  if (m.lin) return m.l;
  auto st = row_major_strides(shape);
  bool aff = true;
  for (const Idx& x : m.co) aff = aff && x.aff;
  if (aff) {
    Idx r = idx_const(d.nd(), 0);
    for (size_t j = 0; j < m.co.size(); ++j) {
      if (shape[j] == 1) continue;
      for (int k = 0; k < d.nd(); ++k) r.c[k] += st[j] * m.co[j].c[k];
      r.k += st[j] * m.co[j].k;
    }
    return r;
  }
  std::string code = "0LL";
  bool o = false, i = false;
  for (size_t j = 0; j < m.co.size(); ++j) {
    if (shape[j] == 1) continue;
    code += "+" + std::to_string(st[j]) + "LL*" + idx_text(m.co[j], d);
    o = o || idx_dep_o(m.co[j], d);
    i = i || idx_dep_i(m.co[j], d);
  }
  return idx_opaque(code, o, i);
}

// Coordinates of a value of shape `shape` read at map m. A linear form is
// decomposed digit-by-digit when every digit term lands inside one
// coordinate without carries (mixed-radix alignment); otherwise div/mod text.
std::vector<Idx> to_coords(const Map& m, const Shape& shape, const Domain& d) {
  if (!m.lin) return m.co;
  const int R = (int)shape.size();
  auto st = row_major_strides(shape);
  std::vector<Idx> out(R, idx_const(d.nd(), 0));
  const Idx& L = m.l;
  bool ok = L.aff && L.k == 0;
  if (ok) {
    std::vector<int64_t> maxv(R, 0);
    for (int k = 0; k < d.nd() && ok; ++k) {
      int64_t c = L.c[k];
      if (!c) continue;
      int64_t ext = k < d.no() ? d.od[k] : d.id[k - d.no()];
      int j = -1;
      for (int t = 0; t < R; ++t) {
        if (shape[t] == 1) continue;
        if (c >= st[t] && c < st[t] * shape[t] && c % st[t] == 0) {
          j = t;
          break;
        }
      }
      if (c < 0 || j < 0) {
        ok = false;
        break;
      }
      out[j].c[k] += c / st[j];
      maxv[j] += (c / st[j]) * (ext - 1);
    }
    for (int j = 0; j < R && ok; ++j)
      if (maxv[j] > shape[j] - 1) ok = false;
  }
  if (ok) return out;
  std::string lt = idx_text(L, d);
  bool o = idx_dep_o(L, d), i = idx_dep_i(L, d);
  for (int j = 0; j < R; ++j) {
    if (shape[j] == 1) continue;
    out[j] = idx_opaque("(" + lt + "/" + std::to_string(st[j]) + "LL)%" + std::to_string(shape[j]) + "LL", o, i);
  }
  return out;
}

bool idx_is_digit(const Idx& a, int digit) {
  if (!a.aff || a.k != 0) return false;
  for (int k = 0; k < (int)a.c.size(); ++k)
    if (a.c[k] != (k == digit ? 1 : 0)) return false;
  return true;
}

// Affine helpers for the index transforms.
static Idx idx_affine(const Idx& a, int64_t scale, int64_t shift, const Domain& d) {
  if (a.aff) {
    Idx r = a;
    for (auto& c : r.c) c *= scale;
    r.k = r.k * scale + shift;
    return r;
  }
  return idx_opaque("(" + idx_text(a, d) + "*" + std::to_string(scale) + "LL+" + std::to_string(shift) + "LL)", a.dep_o,
                    a.dep_i);
}

// A map that carries m's guard (and its digit dependence) plus `cond`.
static Map guarded(Map x, const Map& m, const std::string& cond, bool o, bool i) {
  x.guard = m.guard;
  x.gdep_o = m.gdep_o;
  x.gdep_i = m.gdep_i;
  if (!cond.empty()) {
    x.guard = x.guard.empty() ? cond : "(" + x.guard + ")&&(" + cond + ")";
    x.gdep_o = x.gdep_o || o;
    x.gdep_i = x.gdep_i || i;
  }
  return x;
}

std::string pad_condition(const Graph& g, int id, const Map& m, const Domain& d) {
  const Node& n = g.nodes[id];
  const Node& x = g.nodes[n.args[0]];
  const int r = x.rank();
  auto C = to_coords(m, n.shape, d);
  std::string cond;
  for (int j = 0; j < r; ++j) {
    const int64_t lo = n.attrs[j], inn = n.attrs[r + j], dim = x.shape[j];
    if (lo == 0 && inn == 0 && n.shape[j] == dim) continue;
    const std::string t = "(" + idx_text(C[j], d) + "-" + std::to_string(lo) + "LL)";
    std::string c = t + ">=0LL";
    if (inn == 0) c += "&&" + t + "<" + std::to_string(dim) + "LL";
    else c += "&&" + t + "%" + std::to_string(inn + 1) + "LL==0LL&&" + t + "/" + std::to_string(inn + 1) + "LL<" +
              std::to_string(dim) + "LL";
    cond += (cond.empty() ? "" : "&&") + c;
  }
  return cond;
}

std::string concat_condition(const Graph& g, int id, const Map& m, const Domain& d) {
  const Node& n = g.nodes[id];
  const int ax = (int)n.attrs[0];
  auto C = to_coords(m, n.shape, d);
  return idx_text(C[ax], d) + "<" + std::to_string(g.nodes[n.args[0]].shape[ax]) + "LL";
}

// The gathered index of gather node `id` read at map m, as a variable name
// that the generator declares (fgt_i64) where the gather is evaluated.
std::string gather_index_name(int id, const Map& m) {
  uint64_t h = 1469598103934665603ULL;
  for (char ch : std::to_string(id) + "@" + m.key()) {
    h ^= (unsigned char)ch;
    h *= 1099511628211ULL;
  }
  char b[32];
  std::snprintf(b, sizeof b, "gx%016llx", (unsigned long long)h);
  return b;
}

// Operand maps of a view / elementwise node evaluated at map m.
std::vector<Map> operand_maps(const Graph& g, int id, const Map& m, const Domain& d) {
  const Node& n = g.nodes[id];
  std::vector<Map> r;
  switch (n.op) {
    case FGT_OP_SPLAT:
      r.push_back(guarded(Map{}, m, "", false, false));
      return r;
    case FGT_OP_RESHAPE: {
      Map x;
      x.lin = true;
      x.l = to_linear(m, n.shape, d);
      r.push_back(guarded(x, m, "", false, false));
      return r;
    }
    case FGT_OP_BROADCAST_IN_DIM: {
      auto C = to_coords(m, n.shape, d);
      const Node& x = g.nodes[n.args[0]];
      Map xm;
      for (int a = 0; a < x.rank(); ++a)
        xm.co.push_back(x.shape[a] == 1 ? idx_const(d.nd(), 0) : C[n.attrs[a]]);
      r.push_back(guarded(xm, m, "", false, false));
      return r;
    }
    case FGT_OP_TRANSPOSE: {
      auto C = to_coords(m, n.shape, d);
      const Node& x = g.nodes[n.args[0]];
      Map xm;
      xm.co.assign(x.rank(), idx_const(d.nd(), 0));
      for (int i = 0; i < n.rank(); ++i) xm.co[n.attrs[i]] = C[i];
      r.push_back(guarded(xm, m, "", false, false));
      return r;
    }
    case FGT_OP_SLICE: {
      // operand coordinate = start + step * result coordinate (always in range)
      auto C = to_coords(m, n.shape, d);
      const int rk = n.rank();
      Map xm;
      for (int j = 0; j < rk; ++j) xm.co.push_back(idx_affine(C[j], n.attrs[rk + j], n.attrs[j], d));
      r.push_back(guarded(xm, m, "", false, false));
      return r;
    }
    case FGT_OP_PAD: {
      const Node& x = g.nodes[n.args[0]];
      const int rk = x.rank();
      auto C = to_coords(m, n.shape, d);
      Map xm;
      bool o = false, i = false;
      for (int j = 0; j < rk; ++j) {
        const int64_t lo = n.attrs[j], inn = n.attrs[rk + j];
        const Idx t = idx_affine(C[j], 1, -lo, d);
        if (inn == 0) xm.co.push_back(t);
        else xm.co.push_back(idx_opaque("(" + idx_text(t, d) + "/" + std::to_string(inn + 1) + "LL)", idx_dep_o(t, d),
                                        idx_dep_i(t, d)));
        if (lo != 0 || inn != 0 || n.shape[j] != x.shape[j]) {
          o = o || idx_dep_o(C[j], d);
          i = i || idx_dep_i(C[j], d);
        }
      }
      r.push_back(guarded(xm, m, pad_condition(g, id, m, d), o, i));
      r.push_back(guarded(Map{}, m, "", false, false));  // the rank-0 pad value
      return r;
    }
    case FGT_OP_CONCATENATE: {
      const int ax = (int)n.attrs[0];
      auto C = to_coords(m, n.shape, d);
      const std::string first = concat_condition(g, id, m, d);
      const bool o = idx_dep_o(C[ax], d), i = idx_dep_i(C[ax], d);
      Map am, bm;
      am.co = C;
      bm.co = C;
      bm.co[ax] = idx_affine(C[ax], 1, -g.nodes[n.args[0]].shape[ax], d);
      r.push_back(guarded(am, m, first, o, i));
      r.push_back(guarded(bm, m, "!(" + first + ")", o, i));
      return r;
    }
    case FGT_OP_GATHER: {
      // params[..., indices[i...], ...]; the gathered coordinate is a value
      // (a variable the generator declares), and it may be out of range
      const Node& p = g.nodes[n.args[0]];
      const Node& ix = g.nodes[n.args[1]];
      const int ax = (int)n.attrs[0], ir = ix.rank();
      auto C = to_coords(m, n.shape, d);
      Map im, pm;
      for (int k = 0; k < ir; ++k) im.co.push_back(C[ax + k]);
      const std::string gx = gather_index_name(id, m);
      for (int k = 0; k < ax; ++k) pm.co.push_back(C[k]);
      pm.co.push_back(idx_opaque(gx, true, true));
      for (int k = ax + 1; k < p.rank(); ++k) pm.co.push_back(C[k - 1 + ir]);
      r.push_back(guarded(pm, m, gx + ">=0LL&&" + gx + "<" + std::to_string(p.shape[ax]) + "LL", true, true));
      r.push_back(guarded(im, m, "", false, false));
      return r;
    }
    default:
      for (size_t k = 0; k < n.args.size(); ++k) r.push_back(m);
      return r;
  }
}

// ---------------------------------------------------------------- sharding -
// Leading-dimension sharding: every value carries the axis that is split
// across ranks (or -1). Values that are constant along an axis (splat,
// broadcast-expanded axes) adapt to the local extent; iota along the sharded
// axis gets the rank offset. Reductions over the sharded axis need a
// cross-rank combine; argmax/argmin over it get the rank offset on indices.
Graph shard_graph(const Graph& G, const Options& opt, std::set<int>* combine,
                  std::map<int, int64_t>* index_offsets, std::map<int, int64_t>* iota_offsets) {
  const int W = opt.world;
  Graph g = G;
  const int N = (int)G.nodes.size();
  std::vector<int> axis(N, -1);
  // Pass 1: sharded axis of every value, forward.
  for (int i = 0; i < N; ++i) {
    const Node& n = G.nodes[i];
    auto ax = [&](int k) { return axis[n.args[k]]; };
    switch (n.op) {
      case FGT_OP_PARAMETER:
        if ((opt.shard_inputs >> n.attrs[0]) & 1) {
          require(n.rank() >= 1 && n.shape[0] % W == 0,
                  "sharded input " + std::to_string(n.attrs[0]) + " needs a leading dimension divisible by the world size");
          axis[i] = 0;
        }
        break;
      case FGT_OP_CONSTANT:
      case FGT_OP_SPLAT:
      case FGT_OP_IOTA:
        break;
      case FGT_OP_RESHAPE:
        if (ax(0) >= 0) {
          require(ax(0) == 0 && n.rank() >= 1 && n.shape[0] % W == 0,
                  "reshape of a sharded value must keep a leading dimension divisible by the world size");
          axis[i] = 0;
        }
        break;
      case FGT_OP_BROADCAST_IN_DIM:
        if (ax(0) >= 0) axis[i] = (int)n.attrs[ax(0)];
        break;
      case FGT_OP_TRANSPOSE:
        if (ax(0) >= 0)
          for (int k = 0; k < n.rank(); ++k)
            if (n.attrs[k] == ax(0)) axis[i] = k;
        break;
      case FGT_OP_SLICE:
      case FGT_OP_PAD:
      case FGT_OP_CONCATENATE:
      case FGT_OP_GATHER:
      case FGT_OP_SCATTER_ADD:
        for (size_t k = 0; k < n.args.size(); ++k)
          require(ax((int)k) < 0, std::string(opcode_name(n.op)) + " of a sharded value is not supported", FGT_ERR_UNSUPPORTED);
        break;
      default:
        if (is_reduction(n.op)) {
          if (ax(0) >= 0) {
            auto red = reduced_axes(n);
            if (std::find(red.begin(), red.end(), ax(0)) != red.end()) {
              combine->insert(i);
              if (is_argreduce(n.op)) (*index_offsets)[i] = (int64_t)opt.rank * (G.nodes[n.args[0]].shape[ax(0)] / W);
            } else {
              int before = 0;
              for (int a : red)
                if (a < ax(0)) ++before;
              axis[i] = ax(0) - before;
            }
          }
        } else {
          for (size_t k = 0; k < n.args.size(); ++k) {
            if (ax((int)k) < 0) continue;
            require(axis[i] < 0 || axis[i] == ax((int)k), "operands are sharded along different axes");
            axis[i] = ax((int)k);
          }
        }
    }
  }
  // Pass 2: values consumed by a sharded consumer adopt the local extent,
  // backwards; only values constant along that axis (or iota) may adapt.
  std::vector<int> want(N, -1);
  for (int i = N - 1; i >= 0; --i) {
    const Node& n = G.nodes[i];
    int a = axis[i] >= 0 ? axis[i] : want[i];
    if (a < 0) continue;
    if (axis[i] < 0) {
      // adapting value
      switch (n.op) {
        case FGT_OP_SPLAT:
        case FGT_OP_CONSTANT:
          break;
        case FGT_OP_IOTA:
          if (n.attrs[0] == a) (*iota_offsets)[i] = (int64_t)opt.rank * (n.shape[a] / W);
          break;
        case FGT_OP_BROADCAST_IN_DIM: {
          bool mapped = false;
          for (size_t k = 0; k < n.attrs.size(); ++k)
            if (n.attrs[k] == a && G.nodes[n.args[0]].shape[k] != 1) {
              mapped = true;
              require(want[n.args[0]] < 0 || want[n.args[0]] == (int)k, "conflicting shard axes");
              want[n.args[0]] = (int)k;
            }
          (void)mapped;
          break;
        }
        case FGT_OP_TRANSPOSE:
          want[n.args[0]] = (int)n.attrs[a];
          break;
        case FGT_OP_PARAMETER:
          fail(FGT_ERR_UNSUPPORTED, "an unsharded input is combined elementwise with sharded values");
        default:
          if (is_reduction(n.op) || n.op == FGT_OP_RESHAPE)
            fail(FGT_ERR_UNSUPPORTED, "an unsharded reduction or reshape is combined with sharded values");
          for (int k : n.args) {
            require(want[k] < 0 || want[k] == a, "conflicting shard axes");
            want[k] = a;
          }
      }
    } else if (!is_reduction(n.op) && n.op != FGT_OP_RESHAPE && n.op != FGT_OP_BROADCAST_IN_DIM &&
               n.op != FGT_OP_TRANSPOSE && n.op != FGT_OP_PARAMETER) {
      for (int k : n.args)
        if (axis[k] < 0 && G.nodes[k].rank() > 0) {
          require(want[k] < 0 || want[k] == a, "conflicting shard axes");
          want[k] = a;
        }
    } else if (n.op == FGT_OP_BROADCAST_IN_DIM) {
      // result sharded through its operand: nothing to adapt upstream
    }
  }
  for (int i = 0; i < N; ++i) {
    int a = axis[i] >= 0 ? axis[i] : want[i];
    if (a < 0) continue;
    require(g.nodes[i].shape[a] % W == 0, "sharded extent not divisible by the world size");
    g.nodes[i].shape[a] /= W;
  }
  // Outputs that are split must be produced locally; reductions over the
  // sharded axis are combined and replicated.
  return g;
}

// ------------------------------------------------------- fusibility analysis
static Level join(Level a, Level b) { return Level{a.kind | b.kind, std::max(a.phase, b.phase)}; }

Level Analyzer::of_idx(const Idx& a) {
  Level L;
  if (idx_dep_o(a, d)) L.kind |= 1;
  if (idx_dep_i(a, d)) L.kind |= 2;
  return L;
}

Level Analyzer::run(int id, const Map& m) {
  std::string key = std::to_string(id) + "@" + m.key();
  auto it = memo.find(key);
  if (it != memo.end()) return it->second;
  Level L = compute(id, m);
  memo[key] = L;
  return L;
}

// A reduction computed in this kernel may be read only at its own row (row
// reductions) or, in a FIN kernel, at its own column / as the scalar; any
// other read needs it materialised first.
Level Analyzer::compute(int id, const Map& m) {
  const Node& n = g.nodes[id];
  auto gi = group.find(id);
  if (gi != group.end()) {
    const RedDef& rd = *gi->second;
    auto C = to_coords(m, n.shape, d);
    int digit = 0;
    for (int j = 0; j < n.rank(); ++j) {
      if (n.shape[j] == 1) continue;
      if (!idx_is_digit(C[j], digit)) throw NotFusible{};
      ++digit;
    }
    // In FIN kernels the combined value exists only inside the element loop.
    if (kind == KKind::COLFIN || kind == KKind::FULLFIN) return Level{2, 0};
    if (rd.role != ROLE_ROW) throw NotFusible{};
    Level op = run(n.args[0], rd.opmap);
    red_phase[id] = op.phase;
    return Level{1, op.phase + 1};
  }
  // the kernel that completes a scatter_add computes it (base + accumulator)
  // even once its result has a location
  if (n.op == FGT_OP_SCATTER_ADD && id == finalize_scatter) {
    Level L = run(n.args[0], m);
    return join(L, of_idx(to_linear(m, n.shape, d)));
  }
  if (loc[id].kind != Loc::NONE) {
    const Idx A = to_linear(m, n.shape, d);
    Level L = of_idx(A);
    if (!m.guard.empty()) {
      // a predicated element load is computed where its guard is known
      if (m.gdep_o) L.kind |= 1;
      if (m.gdep_i) L.kind |= 2;
    }
    if (L.kind & 2) {
      loads.insert(id);
      // guarded loads are read one element at a time, and a load that does
      // not move with the innermost digit is read once per chunk: neither
      // limits the vector width
      const bool inner = !A.aff || (d.nd() > 0 && (int)A.c.size() == d.nd() && A.c[d.nd() - 1] != 0);
      if (m.guard.empty() && inner) vec_loads.insert(id);
    }
    return L;
  }
  switch (n.op) {
    case FGT_OP_CONSTANT:
      return Level{};
    case FGT_OP_IOTA: {
      auto C = to_coords(m, n.shape, d);
      return of_idx(C[n.attrs[0]]);
    }
    case FGT_OP_PARAMETER:
      throw NotFusible{};
    default:
      break;
  }
  if (is_reduction(n.op) || n.op == FGT_OP_SCATTER_ADD) throw NotFusible{};
  Level L;
  auto ms = operand_maps(g, id, m, d);
  for (size_t k = 0; k < n.args.size(); ++k) L = join(L, run(n.args[k], ms[k]));
  // pad / concatenate select on coordinates; gather on its index value
  if (n.op == FGT_OP_PAD || n.op == FGT_OP_CONCATENATE || n.op == FGT_OP_GATHER) {
    const Map& gm = ms[0];
    if (gm.gdep_o) L.kind |= 1;
    if (gm.gdep_i) L.kind |= 2;
  }
  return L;
}

// ------------------------------------------------------------------ planner -
namespace {

struct Sig {
  int form = 0;                 // 0 row (reduced digits = I), 1 column (kept = I), 2 full
  std::vector<int64_t> kept, red;  // non-unit extents
};

Sig signature(const Graph& g, int r) {
  const Node& n = g.nodes[r];
  const Node& x = g.nodes[n.args[0]];
  auto axes = reduced_axes(n);
  std::set<int> A(axes.begin(), axes.end());
  Sig s;
  int last = -1;
  for (int j = 0; j < x.rank(); ++j) {
    if (x.shape[j] == 1) continue;
    last = j;
    (A.count(j) ? s.red : s.kept).push_back(x.shape[j]);
  }
  if (s.kept.empty()) s.form = 2;
  else if (last >= 0 && A.count(last)) s.form = 0;
  else s.form = 1;
  return s;
}

// Operand map of reduction r in a domain: its kept axes walk one digit group
// and its reduced axes the other.
Map red_opmap(const Graph& g, int r, const Domain& d, bool kept_are_rows, bool full) {
  const Node& n = g.nodes[r];
  const Node& x = g.nodes[n.args[0]];
  auto axes = reduced_axes(n);
  std::set<int> A(axes.begin(), axes.end());
  Map m;
  if (full) {
    // row-major order over the operand = the domain's element order
    Idx L = idx_const(d.nd(), 0);
    for (int k = 0; k < d.nd(); ++k) L.c[k] = k < d.no() ? d.ow[k] * d.NI : d.iw[k - d.no()];
    m.lin = true;
    m.l = L;
    return m;
  }
  int ko = 0, ki = 0;
  for (int j = 0; j < x.rank(); ++j) {
    if (x.shape[j] == 1) {
      m.co.push_back(idx_const(d.nd(), 0));
      continue;
    }
    bool is_kept = !A.count(j);
    bool row_digit = (is_kept == kept_are_rows);
    if (row_digit) m.co.push_back(idx_digit(d.nd(), ko++));
    else m.co.push_back(idx_digit(d.nd(), d.no() + ki++));
  }
  return m;
}

// Map of a value of `shape` whose non-unit extents are digits [first, first+count).
bool identity_map(const Shape& shape, const Domain& d, int first, int count, Map* out) {
  std::vector<int64_t> ext;
  for (int k = first; k < first + count; ++k) ext.push_back(k < d.no() ? d.od[k] : d.id[k - d.no()]);
  std::vector<int64_t> nu;
  for (int64_t s : shape)
    if (s != 1) nu.push_back(s);
  if (nu != ext) return false;
  Map m;
  int k = first;
  for (int64_t s : shape) m.co.push_back(s == 1 ? idx_const(d.nd(), 0) : idx_digit(d.nd(), k++));
  *out = m;
  return true;
}

int elem_size_of(const Graph& g, int id) { return dtype_size(g.nodes[id].dt); }

struct Planner {
  Graph g;
  Options opt;
  std::set<int> combine;
  std::map<int, int64_t> index_offsets, iota_offsets;
  std::vector<Loc> loc;
  std::set<int> done_outputs;   // output node ids fully stored
  Plan plan;
  int64_t ws = 0;

  Planner(const Graph& g_, const Options& o) : g(g_), opt(o) {}

  int64_t alloc(int64_t bytes) {
    int64_t off = ws;
    ws += (bytes + 255) / 256 * 256;
    return off;
  }

  std::vector<int> output_ports(int node) {
    std::vector<int> p;
    for (size_t k = 0; k < g.outputs.size(); ++k)
      if (g.outputs[k] == node) p.push_back((int)k);
    return p;
  }

  // scatter_add: three ELEM kernels. The accumulator (f64 for floating
  // dtypes, the dtype's own width for integers, whose adds wrap) lives in the
  // workspace; updates at out-of-range indices are dropped
  // (tests/test_stage2_ops.py:230-238).
  void plan_scatter(int s) {
    const Node& n = g.nodes[s];
    const Node& base = g.nodes[n.args[0]];
    const Node& up = g.nodes[n.args[2]];
    const int ax = (int)n.attrs[0], ir = g.nodes[n.args[1]].rank();
    // Bucket form for row scatters whose updates are materialised (read by
    // pointer at any update row): every update is read once and no base-sized
    // accumulator is zeroed, updated atomically and read back. Each base row
    // heads a list of the updates scattered to it.
    const bool csr = ax == 0 && ir == 1 && base.rank() >= 1 && loc[n.args[2]].kind != Loc::NONE && base.shape[0] > 0 &&
                     base.shape[0] < (1LL << 31) && g.nodes[n.args[1]].n() < (1LL << 31);
    const int acc_bytes = is_float(n.dt) ? 8 : dtype_size(n.dt);
    const int64_t R = base.rank() >= 1 ? base.shape[0] : 1, NU = g.nodes[n.args[1]].n();
    // bucket lists: a head per base row (RA = R rounded up to 4 ints, so the
    // next array is 16-byte aligned) and the next update of each index
    const int64_t RA = (R + 3) / 4 * 4;
    const int64_t acc = csr ? alloc((RA + std::max<int64_t>(1, NU)) * 4)
                            : alloc(std::max<int64_t>(1, base.n()) * acc_bytes);
    auto make = [&](const Shape& shape, int stage) {
      KernelDef k;
      k.kind = KKind::ELEM;
      for (int64_t e : shape)
        if (e != 1) k.dom.id.push_back(e);
      k.dom.finish();
      k.scatter_node = s;
      k.scatter_stage = stage;
      k.scatter_acc = acc;
      k.scatter_csr = csr;
      return k;
    };
    auto indices_kernel = [&](int stage) {
      // over the indices: reads indices[i] (any expression of the inputs)
      KernelDef k = make(g.nodes[n.args[1]].shape, stage);
      Analyzer an(g, loc, k.kind, k.dom);
      Map mi;
      mi.lin = true;
      mi.l = idx_const(k.dom.nd(), 0);
      for (int j = 0; j < k.dom.nd(); ++j) mi.l.c[j] = k.dom.iw[j];
      try {
        an.run(n.args[1], mi);
      } catch (NotFusible&) {
        fail(FGT_ERR_UNSUPPORTED, "internal: scatter_add indices not evaluable");
      }
      k.vec = 1;
      geometry_elem(k);
      return k;
    };
    if (csr) {
      KernelDef z = make(Shape{R}, 11);
      z.vec = 1;
      geometry_elem(z);
      plan.kernels.push_back(z);
      if (NU > 0) plan.kernels.push_back(indices_kernel(12));
    }
    auto identity = [&](const KernelDef& k) {
      Map m;
      m.lin = true;
      m.l = idx_const(k.dom.nd(), 0);
      for (int j = 0; j < k.dom.nd(); ++j) m.l.c[j] = k.dom.iw[j];
      return m;
    };
    // 1: accumulator <- 0
    if (!csr) {
      KernelDef k1 = make(base.shape, 1);
      k1.vec = 1;
      geometry_elem(k1);
      plan.kernels.push_back(k1);
    }
    // 2: accumulator[.., indices[i..], ..] += updates[.., i.., ..]
    if (!csr && up.n() > 0) {
      KernelDef k2 = make(up.shape, 2);
      Analyzer an(g, loc, k2.kind, k2.dom);
      const Map mu = identity(k2);
      try {
        an.run(n.args[2], mu);
        auto C = to_coords(mu, up.shape, k2.dom);
        Map mi;
        for (int k = 0; k < ir; ++k) mi.co.push_back(C[ax + k]);
        an.run(n.args[1], mi);
      } catch (NotFusible&) {
        fail(FGT_ERR_UNSUPPORTED, "internal: scatter_add operands not evaluable");
      }
      choose_vec(k2, an.vec_loads, {});
      geometry_elem(k2);
      plan.kernels.push_back(k2);
    }
    // 3: result <- base + accumulator
    KernelDef k3 = make(base.shape, 3);
    Analyzer an(g, loc, k3.kind, k3.dom);
    an.finalize_scatter = s;
    const Map mb = identity(k3);
    try {
      an.run(s, mb);
    } catch (NotFusible&) {
      fail(FGT_ERR_UNSUPPORTED, "internal: scatter_add base not evaluable");
    }
    auto ports = output_ports(s);
    Loc L;
    std::vector<int> outs;
    if (!ports.empty()) {
      L.kind = Loc::OUTPUT;
      L.index = ports[0];
      add_stores(k3, s, 0);
      done_outputs.insert(s);
      outs.push_back(s);
    } else {
      L.kind = Loc::TEMP;
      L.offset = alloc(std::max<int64_t>(1, n.n()) * dtype_size(n.dt));
      OutStore st;
      st.node = s;
      st.port = -1;
      st.temp_offset = L.offset;
      st.level = 0;
      k3.stores.push_back(st);
      outs.push_back(s);
    }
    choose_vec(k3, an.vec_loads, outs);
    geometry_elem(k3);
    // bucket sums: one vector chunk per thread per step, and more resident
    // warps (8 CTAs of 256 per SM) to hide the dependent list loads
    if (csr) k3.unroll = 1;
    plan.kernels.push_back(k3);
    loc[s] = L;
  }

  // Unmaterialised scatter_adds reachable from pending outputs.
  std::vector<int> needed_scatters() {
    std::vector<char> seen(g.nodes.size(), 0);
    std::vector<int> stack;
    for (int o : g.outputs)
      if (!done_outputs.count(o)) stack.push_back(o);
    std::set<int> sc;
    while (!stack.empty()) {
      int id = stack.back();
      stack.pop_back();
      if (seen[id]) continue;
      seen[id] = 1;
      if (loc[id].kind != Loc::NONE) continue;
      if (g.nodes[id].op == FGT_OP_SCATTER_ADD) sc.insert(id);
      for (int a : g.nodes[id].args) stack.push_back(a);
    }
    return std::vector<int>(sc.begin(), sc.end());
  }

  // Unmaterialised reductions reachable from pending outputs, in topo order.
  std::vector<int> needed_reductions() {
    std::vector<char> seen(g.nodes.size(), 0);
    std::vector<int> stack;
    for (int o : g.outputs)
      if (!done_outputs.count(o)) stack.push_back(o);
    std::set<int> reds;
    while (!stack.empty()) {
      int id = stack.back();
      stack.pop_back();
      if (seen[id]) continue;
      seen[id] = 1;
      if (loc[id].kind != Loc::NONE) continue;
      if (is_reduction(g.nodes[id].op)) reds.insert(id);
      for (int a : g.nodes[id].args) stack.push_back(a);
    }
    return std::vector<int>(reds.begin(), reds.end());
  }

  void add_stores(KernelDef& k, int node, int level) {
    auto ports = output_ports(node);
    for (int p : ports) {
      OutStore s;
      s.node = node;
      s.port = p;
      s.level = level;
      k.stores.push_back(s);
    }
  }

  // Element width that sets the vector length of a kernel.
  void choose_vec(KernelDef& k, const std::set<int>& loads, const std::vector<int>& elem_out_nodes) {
    int maxsz = 1;
    for (int id : loads) maxsz = std::max(maxsz, elem_size_of(g, id));
    for (int id : elem_out_nodes) maxsz = std::max(maxsz, elem_size_of(g, id));
    int vec = std::max(1, 16 / maxsz);
    while (vec > 1 && k.dom.NI % vec) vec /= 2;
    k.vec = vec;
  }

  void geometry_row(KernelDef& k) {
    const int64_t NI = k.dom.NI;
    const int64_t nvec = std::max<int64_t>(1, (NI + k.vec - 1) / k.vec);
    // ~row_elems (16) elements per thread per operand: enough independent
    // work per thread, and as many threads per row as that allows (up to 1024).
    const int64_t per_thread_chunks = std::max<int64_t>(1, (opt.row_elems + k.vec - 1) / k.vec);
    if (nvec >= 256) {
      int64_t nt = 128;
      while (nt * 2 <= 1024 && nt * 2 * per_thread_chunks <= nvec) nt *= 2;
      // a row just past nt x 16 chunks takes more threads rather than streaming
      while (nt < 1024 && (nvec + nt - 1) / nt > 16) nt *= 2;
      k.nt = (int)nt;
      k.tpr = (int)nt;
      k.rows_per_cta = 1;
      // A cluster of CTAs shares the row: each CTA holds nt / cluster threads
      // with the same per-thread state, so more rows fit on an SM.
      const int cl = opt.row_cluster;
      if (cl > 1 && nt % cl == 0 && nt / cl >= 64) {
        k.cluster = cl;
        k.nt = (int)(nt / cl);
      }
    } else {
      int64_t tpr = 1;
      while (tpr < 32 && tpr * 2 <= nvec) tpr *= 2;
      k.tpr = (int)tpr;
      k.nt = 256;
      k.rows_per_cta = 256 / tpr;
    }
    k.nch = (int)((nvec + k.tpr - 1) / k.tpr);
    k.streaming = k.nch > 16;
    if (k.streaming) k.nch = (int)((nvec + k.tpr - 1) / k.tpr);
  }

  // Column reductions over rows longer than the register-resident limit: the
  // row splits into column tiles (blockIdx.y), each register-resident with
  // per-thread column accumulators; a CTA walks its rows for one tile, and
  // its partials fill that tile's part of its slots.
  void geometry_tiles(KernelDef& k) {
    const int64_t per_thread_chunks = std::max<int64_t>(1, (opt.row_elems + k.vec - 1) / k.vec);
    k.nt = k.tpr = 256;
    k.rows_per_cta = 1;
    k.cluster = 1;
    k.nch = (int)std::min<int64_t>(16, per_thread_chunks);
    k.tile_elems = (int64_t)k.nt * k.nch * k.vec;
    k.col_tiles = (k.dom.NI + k.tile_elems - 1) / k.tile_elems;
    k.streaming = false;
    if (k.col_tiles > 65535) fail(FGT_ERR_UNSUPPORTED, "column reductions over rows of more than 2^28 elements");
  }

  void geometry_elem(KernelDef& k) {
    k.nt = 256;
    k.tpr = 256;
    k.unroll = 4;
    k.streaming = true;
  }

  void plan_elem_outputs() {
    // Remaining outputs: no unmaterialised reductions remain; one ELEM kernel
    // per distinct element count, domain = the first output's shape.
    std::map<int64_t, std::vector<int>> by_n;
    std::vector<int64_t> order;
    for (int o : g.outputs) {
      if (done_outputs.count(o)) continue;
      int64_t n = g.nodes[o].n();
      if (!by_n.count(n)) order.push_back(n);
      auto& v = by_n[n];
      if (std::find(v.begin(), v.end(), o) == v.end()) v.push_back(o);
    }
    for (int64_t n : order) {
      KernelDef k;
      k.kind = KKind::ELEM;
      const Node& first = g.nodes[by_n[n][0]];
      for (int64_t s : first.shape)
        if (s != 1) k.dom.id.push_back(s);
      k.dom.finish();
      Analyzer an(g, loc, k.kind, k.dom);
      std::vector<int> outs;
      for (int o : by_n[n]) {
        Map m;
        m.lin = true;
        m.l = idx_const(k.dom.nd(), 0);
        for (int j = 0; j < k.dom.nd(); ++j) m.l.c[j] = k.dom.iw[j];
        try {
          an.run(o, m);
        } catch (NotFusible&) {
          fail(FGT_ERR_UNSUPPORTED, "internal: output not evaluable after materialisation");
        }
        add_stores(k, o, 0);
        outs.push_back(o);
        done_outputs.insert(o);
      }
      choose_vec(k, an.vec_loads, outs);
      geometry_elem(k);
      plan.kernels.push_back(k);
    }
  }

  // drop: reductions of this role stay out of the group (later groups take them)
  void plan_group(int r0, int drop = -1) {
    const std::set<int> saved_done = done_outputs;
    const std::vector<Loc> saved_loc = loc;
    const int64_t saved_ws = ws;
    Sig s0 = signature(g, r0);
    KernelDef k;
    k.kind = s0.form == 2 ? KKind::ELEM : KKind::ROW;
    if (s0.form == 0) {
      k.dom.od = s0.kept;
      k.dom.id = s0.red;
    } else if (s0.form == 1) {
      k.dom.od = s0.red;
      k.dom.id = s0.kept;
    } else {
      k.dom.id = s0.red;
    }
    k.dom.finish();
    Analyzer an(g, loc, k.kind, k.dom);
    std::vector<RedDef> reds;
    reds.reserve(g.nodes.size());
    auto R = needed_reductions();
    for (int r : R) {
      Sig s = signature(g, r);
      RedDef rd;
      rd.node = r;
      if (k.kind == KKind::ELEM) {
        if (s.form != 2 || numel(g.nodes[g.nodes[r].args[0]].shape) != k.dom.NI) continue;
        rd.role = ROLE_FULL;
        rd.opmap = red_opmap(g, r, k.dom, false, true);
      } else {
        // Orientation follows which axes are reduced (the signature's form),
        // not extents alone: on square shapes a column reduction also matches
        // the row extents, transposed.
        if (s.form == 0 && s.kept == k.dom.od && s.red == k.dom.id) {
          rd.role = ROLE_ROW;
          rd.opmap = red_opmap(g, r, k.dom, true, false);
        } else if (s.form == 1 && s.kept == k.dom.id && s.red == k.dom.od && !s.kept.empty()) {
          rd.role = ROLE_COL;
          rd.opmap = red_opmap(g, r, k.dom, false, false);
        } else {
          continue;
        }
        if (rd.role == drop) continue;
      }
      if (combine.count(r)) {
        if (rd.role == ROLE_ROW) {
          if (r == r0) fail(FGT_ERR_UNSUPPORTED, "a row-form reduction over the sharded axis is not supported");
          continue;
        }
        rd.combine_ranks = true;
      }
      auto io = index_offsets.find(r);
      if (io != index_offsets.end()) rd.index_offset = io->second;
      reds.push_back(rd);
      an.group[r] = &reds.back();
      an.memo.clear();
      try {
        an.run(g.nodes[r].args[0], rd.opmap);
      } catch (NotFusible&) {
        an.group.erase(r);
        reds.pop_back();
        an.memo.clear();
        if (r == r0) fail(FGT_ERR_UNSUPPORTED, "internal: seed reduction not placeable");
      }
    }
    // Re-run the analysis of the final group to collect loads.
    an.memo.clear();
    an.loads.clear();
    an.vec_loads.clear();
    for (auto& rd : reds) an.run(g.nodes[rd.node].args[0], rd.opmap);
    bool has_col = false, has_full = false;
    for (auto& rd : reds) {
      has_col = has_col || rd.role == ROLE_COL;
      has_full = has_full || rd.role == ROLE_FULL;
    }
    // Outputs placeable in this kernel.
    const Node& seed_x = g.nodes[g.nodes[r0].args[0]];
    std::vector<int> elem_outs;
    std::vector<std::pair<int, int>> fin_outs;  // (node, level)
    for (int o : g.outputs) {
      if (done_outputs.count(o)) continue;
      const Node& on = g.nodes[o];
      bool placed = false;
      auto try_at = [&](const Map& m) {
        try {
          an.run(o, m);
          return true;
        } catch (NotFusible&) {
          return false;
        }
      };
      if (k.kind == KKind::ELEM) {
        if (on.n() == k.dom.NI && on.n() > 1) {
          Map m;
          m.lin = true;
          m.l = idx_const(k.dom.nd(), 0);
          for (int j = 0; j < k.dom.nd(); ++j) m.l.c[j] = k.dom.iw[j];
          if (try_at(m)) {
            add_stores(k, o, 0);
            elem_outs.push_back(o);
            placed = true;
          }
        }
      } else {
        // element level: same non-unit extents as the seed operand
        std::vector<int64_t> a, b;
        for (int64_t s : on.shape)
          if (s != 1) a.push_back(s);
        for (int64_t s : seed_x.shape)
          if (s != 1) b.push_back(s);
        if (a == b && !a.empty()) {
          const Map& sm = reds[0].node == r0 ? reds[0].opmap : an.group[r0]->opmap;
          std::vector<Idx> nu;
          for (size_t j = 0; j < seed_x.shape.size(); ++j)
            if (seed_x.shape[j] != 1) nu.push_back(sm.co[j]);
          Map m;
          size_t t = 0;
          for (int64_t s : on.shape) m.co.push_back(s == 1 ? idx_const(k.dom.nd(), 0) : nu[t++]);
          if (try_at(m)) {
            add_stores(k, o, 0);
            elem_outs.push_back(o);
            placed = true;
          }
        }
        Map m;
        if (!placed && identity_map(on.shape, k.dom, 0, k.dom.no(), &m) && try_at(m)) {
          add_stores(k, o, 1);
          placed = true;
        }
      }
      if (placed) {
        done_outputs.insert(o);
        continue;
      }
      // Column / scalar epilogue outputs are checked against the FIN domain.
      if (has_col || has_full) fin_outs.push_back({o, has_col ? 2 : 3});
    }
    // Materialise the group's reductions.
    for (auto& rd : reds) {
      auto ports = output_ports(rd.node);
      Loc L;
      if (!ports.empty()) {
        L.kind = Loc::OUTPUT;
        L.index = ports[0];
      } else {
        L.kind = Loc::TEMP;
        L.offset = alloc(g.nodes[rd.node].n() * dtype_size(g.nodes[rd.node].dt));
      }
      if (rd.role == ROLE_ROW) {
        if (ports.empty()) {
          OutStore st;
          st.node = rd.node;
          st.port = -1;
          st.temp_offset = L.offset;
          st.level = 1;
          k.stores.push_back(st);
        } else if (!done_outputs.count(rd.node)) {
          add_stores(k, rd.node, 1);
          done_outputs.insert(rd.node);
        }
      }
      loc[rd.node] = L;
    }
    std::vector<int> eo;
    for (auto& st : k.stores)
      if (st.level == 0) eo.push_back(st.node);
    choose_vec(k, an.vec_loads, eo);
    if (k.kind == KKind::ROW) geometry_row(k);
    else geometry_elem(k);
    // Column reductions need register accumulators per element, so not in
    // streaming rows: a group that also holds row reductions is planned again
    // without the role r0 does not have, and a column-only group splits its
    // rows into register-resident column tiles.
    if (k.kind == KKind::ROW && k.streaming && has_col) {
      int r0_role = ROLE_COL;
      bool has_row = false;
      for (auto& rd : reds) {
        if (rd.node == r0) r0_role = rd.role;
        has_row = has_row || rd.role == ROLE_ROW;
      }
      if (has_row) {
        done_outputs = saved_done;
        loc = saved_loc;
        ws = saved_ws;
        plan_group(r0, r0_role == ROLE_COL ? ROLE_ROW : ROLE_COL);
        return;
      }
      geometry_tiles(k);
    }
    k.reds = reds;
    const int kidx = (int)plan.kernels.size();
    plan.kernels.push_back(k);
    if (has_col || has_full) add_fin(kidx, has_col, fin_outs);
  }

  void add_fin(int kidx, bool col, const std::vector<std::pair<int, int>>& fin_outs) {
    KernelDef& prod = plan.kernels[kidx];
    // Partial buffers: one slot per (CTA x row group) of the producer; the
    // launch never uses more CTAs than can be resident at once.
    const int64_t resident =
        std::max<int64_t>(1, (int64_t)opt.num_sms * std::max(1, 2048 / prod.nt) / std::max<int64_t>(1, prod.col_tiles));
    const int64_t units = prod.kind == KKind::ROW ? (prod.dom.NR + prod.rows_per_cta - 1) / prod.rows_per_cta
                                                  : (prod.dom.NI / std::max(1, prod.vec) + prod.nt - 1) / prod.nt;
    prod.max_ctas = std::max<int64_t>(1, std::min(resident, units));
    int64_t slots = prod.max_ctas * (prod.kind == KKind::ROW ? prod.rows_per_cta : 1);
    const int role = col ? ROLE_COL : ROLE_FULL;
    bool any_combine = false;
    for (auto& rd : prod.reds) {
      if (rd.role != role) continue;
      rd.M = col ? prod.dom.NI : 1;
      rd.part_val = alloc(slots * rd.M * 8);
      if (is_argreduce(g.nodes[rd.node].op)) rd.part_idx = alloc(slots * rd.M * 8);
      any_combine = any_combine || rd.combine_ranks;
    }
    KernelDef f;
    f.kind = col ? KKind::COLFIN : KKind::FULLFIN;
    f.producer = kidx;
    if (col) f.dom.id = prod.dom.id;
    f.dom.finish();
    for (auto& rd : prod.reds)
      if (rd.role == role) f.reds.push_back(rd);
    // FIN domain maps of the reductions' results and epilogue outputs.
    Analyzer an(g, loc, f.kind, f.dom);
    std::vector<RedDef> fr = f.reds;
    for (auto& rd : fr) an.group[rd.node] = &rd;
    for (auto& [o, lvl] : fin_outs) {
      if (done_outputs.count(o)) continue;
      const Node& on = g.nodes[o];
      Map m;
      bool ok = col ? identity_map(on.shape, f.dom, 0, f.dom.nd(), &m) : on.n() == 1;
      if (ok && !col) m.co.assign(on.rank(), idx_const(0, 0));
      if (!ok) continue;
      try {
        an.run(o, m);
      } catch (NotFusible&) {
        continue;
      }
      add_stores(f, o, col ? 2 : 3);
      done_outputs.insert(o);
    }
    // The reductions themselves are materialised by the FIN kernel.
    for (auto& rd : f.reds) {
      const Loc& L = loc[rd.node];
      if (L.kind == Loc::TEMP) {
        OutStore st;
        st.node = rd.node;
        st.port = -1;
        st.temp_offset = L.offset;
        st.level = col ? 2 : 3;
        f.stores.push_back(st);
      } else if (!done_outputs.count(rd.node)) {
        add_stores(f, rd.node, col ? 2 : 3);
        done_outputs.insert(rd.node);
      }
    }
    f.nt = 256;
    f.vec = 1;
    if (opt.world > 1 && any_combine) {
      // stage 1: CTA partials -> this rank's record; all-gather; stage 2.
      int64_t rec = 0;
      for (auto& rd : f.reds) rec += rd.M * 8 * (rd.part_idx >= 0 ? 2 : 1);
      KernelDef f1 = f;
      f1.fin_stage = 1;
      f1.stores.clear();
      f1.record_bytes = rec;
      f1.send_offset = alloc(rec);
      f1.recv_offset = alloc(rec * opt.world);
      KernelDef f2 = f;
      f2.fin_stage = 2;
      f2.record_bytes = rec;
      f2.send_offset = f1.send_offset;
      f2.recv_offset = f1.recv_offset;
      f1.path = f2.path = 1;
      plan.kernels.push_back(f1);
      plan.collectives.push_back((int)plan.kernels.size() - 1);
      plan.kernels.push_back(f2);
      // the same two stages in one kernel, the records exchanged through the
      // ranks' peer mailboxes (launched instead when the communicator has them);
      // each 8-byte record value travels as two (value, epoch) words
      if (2 * rec <= kXSlot && opt.world <= kXMaxWorld) {
        KernelDef f3 = f;
        f3.fin_stage = 3;
        f3.record_bytes = rec;
        f3.path = 2;
        plan.kernels.push_back(f3);
      }
    } else {
      plan.kernels.push_back(f);
    }
  }

  Plan run() {
    // The planner works on the local (per-rank) graph.
    if (opt.world > 1) g = shard_graph(g, opt, &combine, &index_offsets, &iota_offsets);
    loc.assign(g.nodes.size(), Loc{});
    for (size_t p = 0; p < g.input_nodes.size(); ++p) {
      loc[g.input_nodes[p]].kind = Loc::INPUT;
      loc[g.input_nodes[p]].index = (int)p;
    }
    for (int guard = 0; guard < 4 * (int)g.nodes.size() + 8; ++guard) {
      bool pending = false;
      for (int o : g.outputs) pending = pending || !done_outputs.count(o);
      if (!pending) break;
      auto R = needed_reductions();
      auto S = needed_scatters();
      // the lowest node first: everything it reads is materialised or fusible
      if (!S.empty() && (R.empty() || S.front() < R.front())) {
        plan_scatter(S.front());
        continue;
      }
      if (R.empty()) {
        plan_elem_outputs();
        break;
      }
      plan_group(R.front());
    }
    for (int o : g.outputs)
      require(done_outputs.count(o), "internal: an output was not planned", FGT_ERR_UNSUPPORTED);
    plan.g = g;
    plan.opt = opt;
    plan.workspace_bytes = ws;
    plan.loc = loc;
    plan.iota_offsets = iota_offsets;
    // Kernel names carry a hash of the partition (nodes, outputs, options), so
    // that launch lists and profiler filters tell the partitions apart.
    uint64_t h = 1469598103934665603ULL;
    auto mix = [&](int64_t v) {
      for (int b = 0; b < 8; ++b) {
        h ^= (uint64_t)((v >> (8 * b)) & 0xff);
        h *= 1099511628211ULL;
      }
    };
    for (const Node& n : g.nodes) {
      mix(n.op);
      mix(n.dt);
      mix(n.pred);
      mix((int64_t)n.cbits);
      for (int64_t e : n.shape) mix(e);
      for (int a : n.args) mix(a);
      for (int64_t a : n.attrs) mix(a);
      mix(-1);
    }
    for (int o : g.outputs) mix(o);
    mix(opt.accumulation);
    mix(opt.world);
    // The rank changes the code only through rank offsets (iota along the
    // split axis, argmax/argmin indices over it); without them every rank's
    // kernels are the same and share one name (and one cached cubin).
    bool rank_offsets = !iota_offsets.empty();
    for (const KernelDef& k : plan.kernels)
      for (const RedDef& rd : k.reds) rank_offsets = rank_offsets || rd.index_offset != 0;
    if (rank_offsets) mix(opt.rank);
    mix(opt.row_elems);
    mix(opt.row_staging);
    mix(opt.lane_pairs);
    mix(opt.own_exp);
    mix(opt.xw_tree);
    mix(opt.smem_cols);
    mix(opt.ring_resident);
    mix(opt.phase_copies);
    mix(opt.pack_cols);
    mix(opt.tmem_cols);
    mix(opt.max3);
    mix(opt.narrow_div);
    mix(opt.occupancy_step);
    mix(opt.ring_kb);
    mix(opt.row_cluster);
    char tag[16];
    std::snprintf(tag, sizeof tag, "%08x", (unsigned)(h ^ (h >> 32)));
    for (size_t i = 0; i < plan.kernels.size(); ++i) {
      KernelDef& k = plan.kernels[i];
      const char* fam = k.kind == KKind::ELEM ? "elem" : k.kind == KKind::ROW ? "row" : k.kind == KKind::COLFIN ? "colfin" : "fullfin";
      k.name = std::string("fgt_") + fam + "_" + std::to_string(i) + "_" + tag;
    }
    return plan;
  }
};

}  // namespace

Plan make_plan(const Graph& g, const Options& opt) {
  Planner p(g, opt);
  return p.run();
}

// ----------------------------------------------------------- plan as JSON ---
static std::string jshape(const Shape& s) {
  std::string r = "[";
  for (size_t i = 0; i < s.size(); ++i) r += (i ? "," : "") + std::to_string(s[i]);
  return r + "]";
}

std::string plan_json(const Plan& plan) {
  const Graph& g = plan.g;
  std::ostringstream j;
  j << "{\"schema_version\":1,\"kind\":\"ask.cuda.execution_plan\",\"inputs\":[";
  for (size_t p = 0; p < g.input_nodes.size(); ++p) j << (p ? "," : "") << "\"in" << p << "\"";
  j << "],\"outputs\":[";
  for (size_t p = 0; p < g.outputs.size(); ++p) j << (p ? "," : "") << "\"out" << p << "\"";
  j << "],\"buffers\":[";
  bool first = true;
  for (size_t p = 0; p < g.input_nodes.size(); ++p) {
    const Node& n = g.nodes[g.input_nodes[p]];
    j << (first ? "" : ",") << "{\"id\":\"in" << p << "\",\"shape\":" << jshape(n.shape) << ",\"element_type\":\""
      << dtype_name(n.dt) << "\"}";
    first = false;
  }
  for (size_t p = 0; p < g.outputs.size(); ++p) {
    const Node& n = g.nodes[g.outputs[p]];
    j << ",{\"id\":\"out" << p << "\",\"shape\":" << jshape(n.shape) << ",\"element_type\":\"" << dtype_name(n.dt)
      << "\"}";
  }
  j << "],\"steps\":[";
  // One owned step per kernel; FIN kernels are steps that read their
  // producer's partials (workspace), so depends_on follows launch order.
  for (size_t i = 0; i < plan.kernels.size(); ++i) {
    const KernelDef& k = plan.kernels[i];
    j << (i ? "," : "") << "{\"id\":\"step" << i << "\",\"kind\":\"owned\",\"function\":\"" << k.name << "\",\"inputs\":[";
    std::set<int> ins;
    for (size_t p = 0; p < g.input_nodes.size(); ++p) ins.insert((int)p);
    bool f = true;
    for (int p : ins) {
      j << (f ? "" : ",") << "\"in" << p << "\"";
      f = false;
    }
    j << "],\"outputs\":[";
    f = true;
    std::set<int> ports;
    for (auto& s : k.stores)
      if (s.port >= 0) ports.insert(s.port);
    for (int p : ports) {
      j << (f ? "" : ",") << "\"out" << p << "\"";
      f = false;
    }
    j << "],\"depends_on\":[";
    if (i > 0) j << "\"step" << (i - 1) << "\"";
    j << "]}";
  }
  j << "],\"scheduling\":{\"policy\":\"sequential\",\"stream\":\"session\"}";
  int loops = 0;
  for (auto& k : plan.kernels) loops += (k.kind == KKind::ELEM || k.kind == KKind::ROW) ? 1 : 0;
  int temps = 0;
  for (auto& k : plan.kernels)
    for (auto& s : k.stores)
      if (s.port < 0) ++temps;
  j << ",\"cuda_lowering\":{\"kernel_count\":" << plan.kernels.size() << ",\"output_loop_count\":" << loops
    << ",\"temporary_buffer_count\":" << temps << ",\"collective_count\":" << plan.collectives.size()
    << ",\"workspace_bytes\":" << plan.workspace_bytes << ",\"kernels\":[";
  for (size_t i = 0; i < plan.kernels.size(); ++i) {
    const KernelDef& k = plan.kernels[i];
    j << (i ? "," : "") << "{\"name\":\"" << k.name << "\",\"rows\":" << k.dom.NR << ",\"row_elements\":" << k.dom.NI
      << ",\"threads\":" << k.nt << ",\"threads_per_row\":" << k.tpr << ",\"cluster\":" << k.cluster
      << ",\"vector\":" << k.vec
      << ",\"chunks\":" << k.nch << ",\"smem_bytes\":" << k.smem_bytes << ",\"streaming\":" << (k.streaming ? "true" : "false")
      << ",\"col_tiles\":" << k.col_tiles
      << ",\"reductions\":" << k.reds.size() << ",\"row_phases\":" << k.row_phases << ",\"registers\":" << k.regs
      << ",\"spill_bytes\":" << k.spill_bytes << "}";
  }
  j << "]}}";
  return j.str();
}

}  // namespace fgt
