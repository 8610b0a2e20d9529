// fgt_plan.h — cutting a partition into fused kernels and specialising each.
//
// Kernel families (every family is a hand-written template in
// fgt_codegen.cpp; what is generated per partition is the element functor,
// the index maps and the reduction set):
//
//   ELEM    grid-stride loop over one iteration domain (flattened), 128-bit
//           vector loads/stores, any number of element outputs, and whole-
//           domain ("full") reductions accumulated per thread -> per-CTA
//           partials.
//   ROW     domain = rows (O digits) x row elements (I digits). One row per
//           lane group (a warp slice, or the whole CTA for long rows); the row
//           is held in registers across phases, so multi-reduction row graphs
//           (softmax, norms, their VJPs) read HBM once. Row reductions (over
//           I) finish with a butterfly + block combine; column reductions
//           (over O) accumulate per thread across the CTA's rows -> partials.
//   COLFIN  combines column partials (CTAs, then ranks), applies the column
//           epilogue (e.g. the bf16 rounding of dgamma) and stores.
//   FULLFIN combines full-reduction partials and applies the scalar epilogue
//           (e.g. mean = sum / count).
//
// The domain of a kernel is a list of "digits" (the non-unit extents of its
// seed reduction's operand, or of its output). Every value evaluated inside a
// kernel carries an index map from digits to its own coordinates; maps are
// affine where the view ops allow it (broadcast, transpose, unit reshapes,
// merges), which is what lets the generator prove a load contiguous and
// vectorise it, or prove that a consumer reads a row reduction at its own row.
#pragma once

#include <map>
#include <set>
#include <string>
#include <vector>

#include "fgt_internal.h"

namespace fgt {

struct Idx {
  bool aff = true;
  std::vector<int64_t> c;  // coefficient per digit (affine form)
  int64_t k = 0;
  std::string code;        // non-affine: C expression (int64)
  bool dep_o = false, dep_i = false;  // for non-affine forms
  std::string key() const;
};

struct Map {
  bool lin = false;          // true: `l` is the value's row-major linear index
  Idx l;
  std::vector<Idx> co;       // false: one coordinate per value dimension
  // Condition (C text over digits and gather indices) under which this
  // value is actually used: set below pad / concatenate / gather, where a
  // coordinate may fall outside its operand. Loads under a guard are element
  // loads predicated on it, never vector loads.
  std::string guard;
  bool gdep_o = false, gdep_i = false;  // digits the guard depends on
  std::string key() const;
};

struct Domain {
  std::vector<int64_t> od, id;   // digit extents: row digits, element digits
  std::vector<int64_t> ow, iw;   // mixed-radix weights within r and e
  int64_t NR = 1, NI = 1;
  int nd() const { return (int)(od.size() + id.size()); }
  int no() const { return (int)od.size(); }
  void finish();
};

enum class KKind { ELEM, ROW, COLFIN, FULLFIN };

// Peer mailbox of one communicator rank: device memory the other ranks'
// processes map through CUDA IPC, zeroed when the communicator is created.
//   epoch           (this rank's own) launches of the exchanging FIN kernels,
//                   with the count of CTAs of the current launch that have
//                   read it in the next word
//   data[par][src]  record words rank src delivered here, each (value,
//                   epoch); par = epoch % 2, so a rank one launch ahead never
//                   overwrites words still read
// A record of one rank for one launch holds at most kXSlot / 2 bytes (its
// words take twice its bytes).
constexpr int kXMaxWorld = 8;
constexpr int kXMaxCtas = 256;
constexpr int64_t kXSlot = 1 << 20;
constexpr int64_t kXEpochOff = 0;
constexpr int64_t kXDataOff = 65536;
constexpr int64_t kXBytes = kXDataOff + 2 * kXMaxWorld * kXSlot;
enum RedRole { ROLE_ROW = 0, ROLE_COL = 1, ROLE_FULL = 2 };

struct RedDef {
  int node = -1;
  int role = ROLE_ROW;
  Map opmap;                 // operand map in the producing kernel's domain
  bool combine_ranks = false;
  int64_t index_offset = 0;  // argmax/argmin on the sharded axis: rank offset
  // partial buffers (COL/FULL): workspace offsets
  int64_t part_val = -1, part_idx = -1;   // [P][M] accumulator / index
  int64_t rank_val = -1, rank_idx = -1;   // gathered [W][M] (sharded)
  int64_t M = 1;                          // partial width (columns or 1)
};

// Where a node's value lives once materialised.
struct Loc {
  enum Kind { NONE, INPUT, OUTPUT, TEMP } kind = NONE;
  int index = -1;        // port index
  int64_t offset = -1;   // workspace byte offset (TEMP)
};

struct OutStore {
  int node = -1;
  int port = -1;         // output port (>=0) or -1 for a temp
  int64_t temp_offset = -1;
  int level = 0;         // 0 element, 1 row, 2 column(fin), 3 scalar(fin)
};

struct KernelDef {
  KKind kind = KKind::ELEM;
  std::string name;
  Domain dom;
  std::vector<RedDef> reds;       // reductions computed (ROW/ELEM) or finalised (FIN)
  std::vector<OutStore> stores;
  int producer = -1;              // FIN kernels: index of the kernel whose partials they read
  int fin_stage = 0;              // FIN: 0 = unsharded, 1 = CTA partials -> rank record, 2 = ranks -> outputs,
                                  // 3 = both with the records exchanged through the peer mailboxes
  int path = 0;                   // sharded specs: 0 always launched, 1 only with NCCL (stages 1, 2),
                                  // 2 only with peer mailboxes (stage 3)
  // geometry (chosen by the planner)
  int nt = 256, tpr = 256, vec = 1, nch = 1, unroll = 1;
  int cluster = 1;                // ROW: CTAs of a thread-block cluster sharing one row (tpr = nt * cluster)
  int64_t col_tiles = 1;          // ROW, column reductions only: the row splits into tiles of tile_elems (blockIdx.y)
  int64_t tile_elems = 0;
  bool streaming = false;
  int64_t rows_per_cta = 1;
  int64_t max_ctas = 0;           // partial slots reserved (grid upper bound)
  int64_t smem_bytes = 0;         // dynamic shared memory (row staging ring)
  int64_t partials = 0;           // P for FIN kernels
  // rank exchange (sharded): record bytes gathered by NCCL after stage 1
  int64_t send_offset = -1, recv_offset = -1, record_bytes = 0;
  std::string source;
  std::string signature;          // human-readable kernel summary
  // scatter_add (ELEM kernels over the base or the updates): stage 1 zeroes
  // the accumulator, 2 adds the in-range updates atomically, 3 combines base
  // and accumulator into the result
  int scatter_node = -1, scatter_stage = 0;
  int64_t scatter_acc = -1;       // workspace offset of the accumulator (CSR: of the row buckets)
  // Row scatter (axis 0, 1-D indices, materialised updates) as a counting
  // sort: 11 zeroes the per-row counters, 12 counts the updates of each base
  // row, 13 scans the counts into bucket offsets (one CTA), 14 fills each
  // row's bucket with its update ids, and 3 sums each output element's bucket
  // in the accumulator type and adds the base (reading every update once).
  bool scatter_csr = false;
  int row_phases = 0;             // ROW: dependency levels holding row reductions (block barriers per row)
  int regs = -1, spill_bytes = -1;  // from the sm_100a compile (-1: unknown)
};

struct Options {
  int accumulation = FGT_ACCUM_WIDE;
  int world = 1, rank = 0;
  uint64_t shard_inputs = 0;
  int num_sms = 148;              // partial buffers are sized for this many SMs
  int max_ctas_per_sm = 8;
  int row_staging = 1;            // next row arrives via cp.async into shared memory (FGT_ROW_STAGING=0: registers)
  int lane_pairs = 1;             // element loops pair lanes for f32x2 arithmetic (FGT_LANE_PAIRS=0: one lane at a time)
  int occupancy_step = 0;         // row kernels: bound registers to fit one more CTA per SM when close (FGT_ROW_OCCUPANCY_STEP)
  int smem_cols = 0;              // row kernels: column accumulators in shared memory (FGT_ROW_SMEM_COLS)
  int xw_tree = 1;                // cross-warp row reductions: tree over the warp partials (FGT_ROW_XW_SHUFFLE: butterfly)
  int own_exp = 1;                // exp in redoable row phases by fgt_exp_q, else expf (FGT_ROW_EXPF, or FGT_OWN_EXP=0)
  int ring_resident = 0;          // row kernels: operands read from the ring in every phase (FGT_ROW_RING_RESIDENT)
  int phase_copies = 0;           // row kernels: later phases read the row operands through opaque copies (FGT_ROW_PHASE_COPIES)
  int pack_cols = 0;              // row kernels: 16-bit per-thread column operands two per register (FGT_ROW_PACK_COLS)
  int tmem_cols = 0;              // row kernels: column accumulators in tensor memory (FGT_ROW_TMEM_COLS)
  int narrow_div = 0;             // row kernels: x * RN(1/d) for divisions of 16-bit-output partitions (FGT_ROW_NARROW_DIV)
  int max3 = 0;                   // three-input max/min for paired range notes (NVRTC >= 12.9; FGT_MAX3=0: off)
  int row_elems = 16;             // elements per thread per row operand in block-per-row kernels (FGT_ROW_ELEMS)
  int ring_kb = 96;               // shared-memory row ring budget per CTA (FGT_RING_KB)
  int row_cluster = 1;            // CTAs per row in block-per-row kernels (thread-block cluster; FGT_ROW_CLUSTER)
};

struct Plan {
  Graph g;                        // local (per-rank) graph
  Options opt;
  std::vector<KernelDef> kernels; // launch order
  std::vector<int> collectives;   // kernel index after which an all-gather runs
  int64_t workspace_bytes = 0;
  std::vector<Loc> loc;                    // final location of materialised nodes
  std::map<int, int64_t> iota_offsets;     // sharded iota: rank offset
};

// ---- index-map algebra shared by the planner and the generator -----------
Idx idx_const(int nd, int64_t v);
Idx idx_digit(int nd, int k);
bool idx_dep_o(const Idx& a, const Domain& d);
bool idx_dep_i(const Idx& a, const Domain& d);
bool idx_is_digit(const Idx& a, int digit);
Idx to_linear(const Map& m, const Shape& shape, const Domain& d);
std::vector<Idx> to_coords(const Map& m, const Shape& shape, const Domain& d);
std::vector<Map> operand_maps(const Graph& g, int id, const Map& m, const Domain& d);
// Conditions of the index transforms at map m (C text): pad / concatenate:
// the value comes from the (first) operand; gather: the index is in range.
std::string pad_condition(const Graph& g, int id, const Map& m, const Domain& d);
std::string concat_condition(const Graph& g, int id, const Map& m, const Domain& d);
std::string gather_index_name(int id, const Map& m);

// Thrown by the analysis when a value cannot be evaluated in a kernel.
struct NotFusible {};

// Where in a kernel a value can first be computed.
struct Level {
  int kind = 0;   // bit0: varies with the row, bit1: varies within the row
  int phase = 0;  // element-loop index from which the value is computable
};

// Fusibility / placement analysis of values inside one kernel.
struct Analyzer {
  const Graph& g;
  const std::vector<Loc>& loc;
  KKind kind;
  int finalize_scatter = -1;      // the scatter_add node this kernel completes (read as base + accumulator)
  const Domain& d;
  std::map<int, const RedDef*> group;  // reductions computed (or finalised) here
  std::map<std::string, Level> memo;
  std::map<int, int> red_phase;        // row reduction -> element loop it runs in
  std::set<int> loads;                 // nodes loaded with in-row dependence
  std::set<int> vec_loads;             // of those, the unguarded ones whose address moves with the innermost
                                       // digit: the only loads that may be read as vectors
  Analyzer(const Graph& g_, const std::vector<Loc>& l, KKind k, const Domain& d_) : g(g_), loc(l), kind(k), d(d_) {}
  Level run(int id, const Map& m);

 private:
  Level compute(int id, const Map& m);
  Level of_idx(const Idx& a);
};

// Shard the global graph for (rank, world): local shapes, rank offsets and
// the reductions that need a cross-rank combine.
Graph shard_graph(const Graph& global, const Options& opt, std::set<int>* combine,
                  std::map<int, int64_t>* index_offsets, std::map<int, int64_t>* iota_offsets);

Plan make_plan(const Graph& g, const Options& opt);

// Emit CUDA source for every kernel of the plan.
void generate_sources(Plan& plan);

std::string plan_json(const Plan& plan);

}  // namespace fgt
