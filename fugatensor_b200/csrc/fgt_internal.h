// fgt_internal.h — internal IR of a partition and shared helpers.
#pragma once

#include <cstdint>
#include <stdexcept>
#include <string>
#include <vector>

#include "fgt.h"

namespace fgt {

// Error carried to the C ABI as (status, message).
struct Error : std::runtime_error {
  fgt_status status;
  Error(fgt_status s, const std::string& m) : std::runtime_error(m), status(s) {}
};
[[noreturn]] inline void fail(fgt_status s, const std::string& m) { throw Error(s, m); }
inline void require(bool ok, const std::string& m, fgt_status s = FGT_ERR_INVALID) {
  if (!ok) fail(s, m);
}

using Shape = std::vector<int64_t>;

inline int64_t numel(const Shape& s) {
  int64_t n = 1;
  for (int64_t d : s) n *= d;
  return n;
}
inline std::vector<int64_t> row_major_strides(const Shape& s) {
  std::vector<int64_t> st(s.size(), 1);
  for (int i = (int)s.size() - 2; i >= 0; --i) st[i] = st[i + 1] * s[i + 1];
  return st;
}

inline int dtype_size(int dt) {
  switch (dt) {
    case FGT_BOOL: return 1;
    case FGT_I32: return 4;
    case FGT_I64: return 8;
    case FGT_F32: return 4;
    case FGT_F16: return 2;
    case FGT_BF16: return 2;
  }
  return 0;
}
inline bool is_float(int dt) { return dt == FGT_F32 || dt == FGT_F16 || dt == FGT_BF16; }
inline bool is_int(int dt) { return dt == FGT_I32 || dt == FGT_I64; }
inline const char* dtype_name(int dt) {
  switch (dt) {
    case FGT_BOOL: return "bool";
    case FGT_I32: return "i32";
    case FGT_I64: return "i64";
    case FGT_F32: return "f32";
    case FGT_F16: return "f16";
    case FGT_BF16: return "bf16";
  }
  return "?";
}
const char* opcode_name(int op);

inline bool is_reduction(int op) {
  return op >= FGT_OP_REDUCE_SUM && op <= FGT_OP_ARGMIN;
}
inline bool is_argreduce(int op) { return op == FGT_OP_ARGMAX || op == FGT_OP_ARGMIN; }
inline bool is_binary(int op) { return op >= FGT_OP_ADD && op <= FGT_OP_SHIFT_RIGHT; }
inline bool is_unary(int op) { return op >= FGT_OP_EXP && op <= FGT_OP_BITWISE_NOT; }

struct Node {
  int op = 0;
  int dt = 0;
  Shape shape;
  std::vector<int> args;
  std::vector<int64_t> attrs;
  int pred = 0;
  uint64_t cbits = 0;
  int64_t n() const { return numel(shape); }
  int rank() const { return (int)shape.size(); }
};

struct Graph {
  std::vector<Node> nodes;
  std::vector<int> outputs;      // node ids in output port order
  std::vector<int> input_nodes;  // node id per input port
  std::vector<std::vector<int>> users;
};

// Build and type-check a graph from the C descriptor (Fuga typing rules).
Graph build_graph(const fgt_partition_desc* desc);

// Reduced axes of a reduction node (argmax/argmin: its single axis).
std::vector<int> reduced_axes(const Node& n);

}  // namespace fgt
