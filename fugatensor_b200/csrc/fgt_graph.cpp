// fgt_graph.cpp — partition descriptor -> checked IR.
//
// Every node's declared type must equal the type Fuga's abstract evaluation
// infers (src/fugatensor/ir/primitives.py:186-199 validate_primitive), with the
// rules of src/fugatensor/ir/tensor_rules.py and primitives.py:
//   arithmetic add/mul: matching operands, no bool (primitives.py:80-85);
//   div / transcendentals / rounding: floating only (tensor_rules.py:170,184-186);
//   compare: matching operands -> bool (tensor_rules.py:26-31);
//   select: bool condition of the value shape, matching values (:34-37);
//   broadcast_in_dim: increasing dims, size-1 expansion only (:40-52);
//   transpose: a permutation (:55-62);
//   reductions: sorted unique axes, non-bool (any/all: bool), max/min
//   nonempty (:65-92); argmax/argmin: one axis, nonempty, i64 (:95-108).
#include <algorithm>
#include <set>

#include "fgt_internal.h"

namespace fgt {

const char* opcode_name(int op) {
  switch (op) {
    case FGT_OP_PARAMETER: return "parameter";
    case FGT_OP_CONSTANT: return "constant";
    case FGT_OP_SPLAT: return "splat";
    case FGT_OP_RESHAPE: return "reshape";
    case FGT_OP_BROADCAST_IN_DIM: return "broadcast_in_dim";
    case FGT_OP_TRANSPOSE: return "transpose";
    case FGT_OP_STOP_GRADIENT: return "stop_gradient";
    case FGT_OP_IOTA: return "iota";
    case FGT_OP_CAST: return "cast";
    case FGT_OP_ADD: return "add";
    case FGT_OP_MUL: return "mul";
    case FGT_OP_DIV: return "div";
    case FGT_OP_MAXIMUM: return "maximum";
    case FGT_OP_MINIMUM: return "minimum";
    case FGT_OP_POW: return "pow";
    case FGT_OP_FLOORDIV: return "floordiv";
    case FGT_OP_MOD: return "mod";
    case FGT_OP_BITWISE_AND: return "bitwise_and";
    case FGT_OP_BITWISE_OR: return "bitwise_or";
    case FGT_OP_BITWISE_XOR: return "bitwise_xor";
    case FGT_OP_SHIFT_LEFT: return "shift_left";
    case FGT_OP_SHIFT_RIGHT: return "shift_right";
    case FGT_OP_EXP: return "exp";
    case FGT_OP_LOG: return "log";
    case FGT_OP_SQRT: return "sqrt";
    case FGT_OP_SIN: return "sin";
    case FGT_OP_COS: return "cos";
    case FGT_OP_TANH: return "tanh";
    case FGT_OP_ERF: return "erf";
    case FGT_OP_ABS: return "abs";
    case FGT_OP_FLOOR: return "floor";
    case FGT_OP_CEIL: return "ceil";
    case FGT_OP_ROUND: return "round";
    case FGT_OP_BITWISE_NOT: return "bitwise_not";
    case FGT_OP_COMPARE: return "compare";
    case FGT_OP_SELECT: return "select";
    case FGT_OP_REDUCE_SUM: return "reduce_sum";
    case FGT_OP_REDUCE_MAX: return "reduce_max";
    case FGT_OP_REDUCE_MIN: return "reduce_min";
    case FGT_OP_REDUCE_PROD: return "reduce_prod";
    case FGT_OP_REDUCE_ANY: return "reduce_any";
    case FGT_OP_REDUCE_ALL: return "reduce_all";
    case FGT_OP_ARGMAX: return "argmax";
    case FGT_OP_ARGMIN: return "argmin";
    case FGT_OP_SLICE: return "slice";
    case FGT_OP_PAD: return "pad";
    case FGT_OP_CONCATENATE: return "concatenate";
    case FGT_OP_GATHER: return "gather";
    case FGT_OP_SCATTER_ADD: return "scatter_add";
  }
  return "unknown";
}

std::vector<int> reduced_axes(const Node& n) {
  std::vector<int> axes;
  for (int64_t a : n.attrs) axes.push_back((int)a);
  return axes;
}

namespace {

bool valid_dtype(int dt) { return dt >= FGT_BOOL && dt <= FGT_BF16; }
bool valid_opcode(int op) {
  return (op >= FGT_OP_PARAMETER && op <= FGT_OP_CAST) || (op >= FGT_OP_ADD && op <= FGT_OP_SHIFT_RIGHT) ||
         (op >= FGT_OP_EXP && op <= FGT_OP_BITWISE_NOT) || op == FGT_OP_COMPARE || op == FGT_OP_SELECT ||
         (op >= FGT_OP_REDUCE_SUM && op <= FGT_OP_ARGMIN) || (op >= FGT_OP_SLICE && op <= FGT_OP_SCATTER_ADD);
}

std::string where(int id, const Node& n) {
  return "node " + std::to_string(id) + " (" + opcode_name(n.op) + ")";
}

void infer(const Graph& g, int id) {
  const Node& n = g.nodes[id];
  auto arg = [&](int k) -> const Node& { return g.nodes[n.args[k]]; };
  auto nargs = [&](size_t k) {
    require(n.args.size() == k, where(id, n) + ": expects " + std::to_string(k) + " operands");
  };
  auto same_as = [&](const Node& o) {
    require(n.dt == o.dt && n.shape == o.shape, where(id, n) + ": result type must match its operand");
  };
  const std::string w = where(id, n);
  switch (n.op) {
    case FGT_OP_PARAMETER:
      nargs(0);
      require(n.attrs.size() == 1, w + ": parameter needs its input port index in attrs[0]");
      return;
    case FGT_OP_CONSTANT:
      nargs(0);
      require(n.shape.empty(), w + ": constants are rank 0 (use splat)");
      return;
    case FGT_OP_SPLAT:
      nargs(1);
      require(arg(0).shape.empty() && arg(0).dt == n.dt, w + ": splat takes a rank-0 operand of its dtype");
      return;
    case FGT_OP_RESHAPE:
      nargs(1);
      require(arg(0).dt == n.dt && arg(0).n() == n.n(), w + ": reshape must keep dtype and element count");
      return;
    case FGT_OP_BROADCAST_IN_DIM: {
      nargs(1);
      const Node& x = arg(0);
      require(x.dt == n.dt, w + ": broadcast keeps dtype");
      require((int)n.attrs.size() == x.rank(), w + ": broadcast dimensions must map every operand axis");
      for (size_t k = 0; k < n.attrs.size(); ++k) {
        int64_t d = n.attrs[k];
        require(d >= 0 && d < n.rank(), w + ": broadcast dimension out of range");
        require(k == 0 || n.attrs[k - 1] < d, w + ": broadcast dimensions must be increasing");
        require(x.shape[k] == 1 || x.shape[k] == n.shape[d], w + ": broadcast mapped dimensions must match or have size one");
      }
      return;
    }
    case FGT_OP_TRANSPOSE: {
      nargs(1);
      const Node& x = arg(0);
      require(x.dt == n.dt && (int)n.attrs.size() == x.rank(), w + ": transpose needs a full permutation");
      std::vector<int64_t> p = n.attrs;
      std::sort(p.begin(), p.end());
      for (int k = 0; k < x.rank(); ++k) require(p[k] == k, w + ": transpose permutation must contain each axis once");
      for (int k = 0; k < x.rank(); ++k)
        require(n.shape[k] == x.shape[n.attrs[k]], w + ": transpose result shape mismatch");
      return;
    }
    case FGT_OP_STOP_GRADIENT:
      nargs(1);
      same_as(arg(0));
      return;
    case FGT_OP_IOTA:
      nargs(0);
      require(n.rank() >= 1 && n.attrs.size() == 1 && n.attrs[0] >= 0 && n.attrs[0] < n.rank(),
              w + ": iota needs rank >= 1 and a dimension in range");
      require(n.dt != FGT_BOOL, w + ": iota requires a numeric dtype");
      return;
    case FGT_OP_CAST:
      nargs(1);
      require(arg(0).shape == n.shape, w + ": cast keeps the shape");
      return;
    case FGT_OP_COMPARE:
      nargs(2);
      require(arg(0).dt == arg(1).dt && arg(0).shape == arg(1).shape, w + ": compare requires matching operand types");
      require(n.dt == FGT_BOOL && n.shape == arg(0).shape, w + ": compare yields bool of the operand shape");
      require(n.pred >= FGT_CMP_EQ && n.pred <= FGT_CMP_GE, w + ": compare predicate must be eq/ne/lt/le/gt/ge");
      return;
    case FGT_OP_SELECT:
      nargs(3);
      require(arg(0).dt == FGT_BOOL && arg(0).shape == arg(1).shape, w + ": select requires a bool condition of the value shape");
      require(arg(1).dt == arg(2).dt && arg(1).shape == arg(2).shape, w + ": select values must match");
      same_as(arg(1));
      return;
    // index transforms: ir/tensor_rules.py:124-237
    case FGT_OP_SLICE: {
      nargs(1);
      const Node& x = arg(0);
      const int r = x.rank();
      require(x.dt == n.dt && n.rank() == r && (int)n.attrs.size() == 2 * r, w + ": slice needs starts and steps per axis");
      for (int j = 0; j < r; ++j) {
        const int64_t st = n.attrs[j], step = n.attrs[r + j], out = n.shape[j], dim = x.shape[j];
        require(step != 0, w + ": slice step must be nonzero");
        require(out >= 0, w + ": slice extent");
        if (out == 0) continue;
        const int64_t last = st + (out - 1) * step;
        require(st >= 0 && st < dim && last >= 0 && last < dim, w + ": slice bounds out of range");
      }
      return;
    }
    case FGT_OP_PAD: {
      nargs(2);
      const Node& x = arg(0);
      const int r = x.rank();
      require(arg(1).shape.empty() && arg(1).dt == x.dt && n.dt == x.dt,
              w + ": pad requires a 0-D scalar pad_value with the same dtype as input");
      require(n.rank() == r && (int)n.attrs.size() == 2 * r, w + ": pad needs low and interior per axis");
      for (int j = 0; j < r; ++j) {
        const int64_t lo = n.attrs[j], inn = n.attrs[r + j], dim = x.shape[j];
        require(lo >= 0 && inn >= 0, w + ": pad amounts and interior dilation must be nonnegative");
        const int64_t inner = dim > 0 ? dim + (dim - 1) * inn : 0;
        require(n.shape[j] >= lo + inner, w + ": pad high must be nonnegative");
      }
      return;
    }
    case FGT_OP_CONCATENATE: {
      nargs(2);
      const Node &a = arg(0), &b = arg(1);
      require(n.attrs.size() == 1 && a.rank() >= 1 && n.attrs[0] >= 0 && n.attrs[0] < a.rank(),
              w + ": concatenate axis out of range");
      require(a.dt == b.dt && a.rank() == b.rank() && n.dt == a.dt && n.rank() == a.rank(),
              w + ": concatenate operands must match rank and dtype");
      const int ax = (int)n.attrs[0];
      for (int j = 0; j < a.rank(); ++j)
        require(j == ax ? n.shape[j] == a.shape[j] + b.shape[j] : (a.shape[j] == b.shape[j] && n.shape[j] == a.shape[j]),
                w + ": concatenate non-axis dimensions must match");
      return;
    }
    case FGT_OP_GATHER: {
      nargs(2);
      const Node &p = arg(0), &ix = arg(1);
      require(p.rank() >= 1 && n.attrs.size() == 1 && n.attrs[0] >= 0 && n.attrs[0] < p.rank(),
              w + ": gather axis out of range");
      require(is_int(ix.dt), w + ": gather indices must have i32 or i64 dtype");
      const int ax = (int)n.attrs[0];
      Shape want(p.shape.begin(), p.shape.begin() + ax);
      want.insert(want.end(), ix.shape.begin(), ix.shape.end());
      want.insert(want.end(), p.shape.begin() + ax + 1, p.shape.end());
      require(n.dt == p.dt && n.shape == want, w + ": gather result type mismatch");
      return;
    }
    case FGT_OP_SCATTER_ADD: {
      nargs(3);
      const Node &b = arg(0), &ix = arg(1), &u = arg(2);
      require(b.rank() >= 1 && n.attrs.size() == 1 && n.attrs[0] >= 0 && n.attrs[0] < b.rank(),
              w + ": scatter_add axis out of range");
      require(b.dt != FGT_BOOL, w + ": scatter_add base must have a numeric dtype");
      require(is_int(ix.dt), w + ": scatter_add indices must have i32 or i64 type");
      const int ax = (int)n.attrs[0];
      Shape want(b.shape.begin(), b.shape.begin() + ax);
      want.insert(want.end(), ix.shape.begin(), ix.shape.end());
      want.insert(want.end(), b.shape.begin() + ax + 1, b.shape.end());
      require(u.dt == b.dt && u.shape == want, w + ": scatter_add updates shape/dtype does not match base, indices and axis");
      same_as(b);
      return;
    }
    default:
      break;
  }
  if (is_binary(n.op)) {
    nargs(2);
    require(arg(0).dt == arg(1).dt && arg(0).shape == arg(1).shape,
            w + ": operation requires matching operands (no implicit broadcast)");
    same_as(arg(0));
    switch (n.op) {
      case FGT_OP_ADD:
      case FGT_OP_MUL:
      case FGT_OP_POW:
      case FGT_OP_FLOORDIV:
      case FGT_OP_MOD:
        require(n.dt != FGT_BOOL, w + ": bool arithmetic is undefined");
        break;
      case FGT_OP_DIV:
        require(is_float(n.dt), w + ": div is floating division");
        break;
      case FGT_OP_BITWISE_AND:
      case FGT_OP_BITWISE_OR:
      case FGT_OP_BITWISE_XOR:
        require(!is_float(n.dt), w + ": bitwise operations take integer or bool operands");
        break;
      case FGT_OP_SHIFT_LEFT:
      case FGT_OP_SHIFT_RIGHT:
        require(is_int(n.dt), w + ": shifts take integer operands");
        break;
      default:
        break;
    }
    return;
  }
  if (is_unary(n.op)) {
    nargs(1);
    same_as(arg(0));
    if (n.op == FGT_OP_ABS) require(n.dt != FGT_BOOL, w + ": abs requires a numeric dtype");
    else if (n.op == FGT_OP_BITWISE_NOT) require(!is_float(n.dt), w + ": bitwise_not takes integer or bool");
    else require(is_float(n.dt), w + ": unsupported dtype for a floating operation");
    return;
  }
  if (is_reduction(n.op)) {
    nargs(1);
    const Node& x = arg(0);
    if (is_argreduce(n.op)) {
      require(n.attrs.size() == 1, w + ": argmax/argmin requires one integer axis");
      int64_t a = n.attrs[0];
      require(x.rank() >= 1 && a >= 0 && a < x.rank(), w + ": argmax/argmin axis out of range");
      require(x.shape[a] > 0, w + ": argmax/argmin requires a nonempty reduction domain");
      require(x.dt != FGT_BOOL, w + ": argmax/argmin requires a numeric operand");
      require(n.dt == FGT_I64, w + ": argmax/argmin yields i64");
      Shape rest;
      for (int k = 0; k < x.rank(); ++k)
        if (k != a) rest.push_back(x.shape[k]);
      require(n.shape == rest, w + ": argmax/argmin result shape mismatch");
      return;
    }
    bool boolean = n.op == FGT_OP_REDUCE_ANY || n.op == FGT_OP_REDUCE_ALL;
    require(boolean ? x.dt == FGT_BOOL : x.dt != FGT_BOOL,
            boolean ? w + ": boolean reduction requires a bool operand" : w + ": reduction requires a numeric operand");
    for (size_t k = 0; k < n.attrs.size(); ++k) {
      require(n.attrs[k] >= 0 && n.attrs[k] < x.rank() && (k == 0 || n.attrs[k - 1] < n.attrs[k]),
              w + ": reduction axes must be sorted, unique and in range");
    }
    std::set<int64_t> axes(n.attrs.begin(), n.attrs.end());
    if (n.op == FGT_OP_REDUCE_MAX || n.op == FGT_OP_REDUCE_MIN)
      for (int64_t a : axes) require(x.shape[a] > 0, w + ": max/min reduction requires a nonempty reduction domain");
    Shape rest;
    for (int k = 0; k < x.rank(); ++k)
      if (!axes.count(k)) rest.push_back(x.shape[k]);
    require(n.dt == x.dt && n.shape == rest, w + ": reduction result type mismatch");
    return;
  }
  fail(FGT_ERR_UNSUPPORTED, w + ": opcode not supported");
}

}  // namespace

Graph build_graph(const fgt_partition_desc* desc) {
  require(desc != nullptr, "partition descriptor is NULL");
  require(desc->abi_version == FGT_ABI_VERSION, "partition descriptor ABI version mismatch");
  require(desc->num_nodes > 0 && desc->nodes != nullptr, "partition has no nodes");
  require(desc->num_outputs > 0 && desc->outputs != nullptr, "partition requires at least one output");
  Graph g;
  g.nodes.resize(desc->num_nodes);
  int max_port = -1;
  for (int i = 0; i < desc->num_nodes; ++i) {
    const fgt_node& s = desc->nodes[i];
    Node& n = g.nodes[i];
    require(valid_opcode(s.opcode), "node " + std::to_string(i) + ": unknown opcode " + std::to_string(s.opcode));
    require(valid_dtype(s.dtype), "node " + std::to_string(i) + ": unknown dtype");
    require(s.rank >= 0 && s.rank <= FGT_MAX_RANK, "node " + std::to_string(i) + ": rank out of range");
    require(s.num_operands >= 0 && s.num_operands <= FGT_MAX_OPERANDS, "node " + std::to_string(i) + ": operand count");
    require(s.num_attrs >= 0 && s.num_attrs <= FGT_MAX_ATTRS, "node " + std::to_string(i) + ": attr count");
    n.op = s.opcode;
    n.dt = s.dtype;
    for (int k = 0; k < s.rank; ++k) {
      require(s.shape[k] >= 0, "node " + std::to_string(i) + ": negative extent");
      n.shape.push_back(s.shape[k]);
    }
    for (int k = 0; k < s.num_operands; ++k) {
      int a = s.operands[k];
      require(a >= 0 && a < i, "node " + std::to_string(i) + ": operands must name earlier nodes");
      n.args.push_back(a);
    }
    for (int k = 0; k < s.num_attrs; ++k) n.attrs.push_back(s.attrs[k]);
    n.pred = s.predicate;
    n.cbits = s.constant_bits;
    infer(g, i);
    if (n.op == FGT_OP_PARAMETER) {
      int port = (int)n.attrs[0];
      require(port >= 0 && port < 64, "parameter port index out of range");
      if ((int)g.input_nodes.size() <= port) g.input_nodes.resize(port + 1, -1);
      require(g.input_nodes[port] == -1, "input port " + std::to_string(port) + " is bound twice");
      g.input_nodes[port] = i;
      max_port = std::max(max_port, port);
    }
  }
  for (size_t p = 0; p < g.input_nodes.size(); ++p)
    require(g.input_nodes[p] >= 0, "input ports must be numbered densely from 0");
  for (int k = 0; k < desc->num_outputs; ++k) {
    int o = desc->outputs[k];
    require(o >= 0 && o < desc->num_nodes, "output names an unknown node");
    g.outputs.push_back(o);
  }
  g.users.assign(g.nodes.size(), {});
  for (size_t i = 0; i < g.nodes.size(); ++i)
    for (int a : g.nodes[i].args) g.users[a].push_back((int)i);
  return g;
}

}  // namespace fgt
