/*
 * fgt.h — C ABI of the B200-native (sm_100a) backend for FugaTensor's fused
 * elementwise / broadcast / reduction partitions.
 *
 * A partition is a small SSA DAG of Fuga primitives (the ops that the
 * reference lowers to ASK "owned" kernels, src/fugatensor/lowering.py:88-111).
 * The caller describes it with plain C structs; the library type-checks it
 * with Fuga's typing rules (src/fugatensor/ir/tensor_rules.py,
 * src/fugatensor/ir/primitives.py), cuts it into fused kernels, specialises a
 * hand-written sm_100a kernel template per kernel (dtype, rank, broadcast
 * pattern, reduce axis), compiles it once and launches it on a caller stream.
 *
 * Conventions (kept from the reference runtime, cpp/ask_runtime.cpp:18-24,
 * src/fugatensor/_ask/cuda.py:118):
 *   - dtypes bool/i32/i64/f32/f16/bf16, widths 1/4/8/4/2/2 bytes;
 *   - every buffer is dense, contiguous, row-major; shapes are static;
 *     0-D and empty tensors are allowed;
 *   - buffers are caller-owned device memory; the library allocates nothing
 *     on the launch path (scratch lives in a caller-provided workspace);
 *   - statuses are integers; no exception crosses the ABI; the message of the
 *     last failure on the calling thread is returned by fgt_last_error();
 *   - validation happens before any launch; there is no CPU fallback.
 *
 * No torch types appear here: a cgo / ctypes / JNI caller binds this header
 * directly.
 */
#ifndef FGT_H_
#define FGT_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FGT_ABI_VERSION 5
#define FGT_MAX_RANK 8
#define FGT_MAX_OPERANDS 3
#define FGT_MAX_ATTRS 24

typedef int32_t fgt_status;
enum {
  FGT_OK = 0,
  FGT_ERR_INVALID = 1,      /* malformed descriptor, type error, bad argument   */
  FGT_ERR_UNSUPPORTED = 2,  /* well-formed but outside what the backend plans   */
  FGT_ERR_COMPILE = 3,      /* kernel specialisation failed to compile          */
  FGT_ERR_CUDA = 4,         /* a CUDA driver call failed                         */
  FGT_ERR_NCCL = 5,         /* a collective failed or timed out                  */
  FGT_ERR_WORKSPACE = 6     /* workspace missing or smaller than required        */
};

/* Element types; numbering is part of the ABI. */
typedef enum fgt_dtype {
  FGT_BOOL = 0, FGT_I32 = 1, FGT_I64 = 2, FGT_F32 = 3, FGT_F16 = 4, FGT_BF16 = 5
} fgt_dtype;

/* Opcodes: one per Fuga primitive on the path. Numbering is part of the ABI. */
typedef enum fgt_opcode {
  /* leaves and views */
  FGT_OP_PARAMETER = 0,       /* attrs[0] = input port index                           */
  FGT_OP_CONSTANT = 1,        /* rank 0; constant_bits = value in dtype's encoding     */
  FGT_OP_SPLAT = 2,           /* rank-0 operand -> shape                               */
  FGT_OP_RESHAPE = 3,         /* same element count, row-major relinearisation         */
  FGT_OP_BROADCAST_IN_DIM = 4,/* attrs = dimensions (operand axis -> result axis)      */
  FGT_OP_TRANSPOSE = 5,       /* attrs = permutation                                   */
  FGT_OP_STOP_GRADIENT = 6,   /* identity                                              */
  FGT_OP_IOTA = 7,            /* attrs[0] = dimension                                  */
  FGT_OP_CAST = 8,            /* dtype conversion (saturating float->int, NaN->0)      */
  /* binary elementwise (operands: equal shape and dtype) */
  FGT_OP_ADD = 10, FGT_OP_MUL = 11, FGT_OP_DIV = 12, FGT_OP_MAXIMUM = 13,
  FGT_OP_MINIMUM = 14, FGT_OP_POW = 15, FGT_OP_FLOORDIV = 16, FGT_OP_MOD = 17,
  FGT_OP_BITWISE_AND = 18, FGT_OP_BITWISE_OR = 19, FGT_OP_BITWISE_XOR = 20,
  FGT_OP_SHIFT_LEFT = 21, FGT_OP_SHIFT_RIGHT = 22,
  /* unary elementwise */
  FGT_OP_EXP = 30, FGT_OP_LOG = 31, FGT_OP_SQRT = 32, FGT_OP_SIN = 33, FGT_OP_COS = 34,
  FGT_OP_TANH = 35, FGT_OP_ERF = 36, FGT_OP_ABS = 37, FGT_OP_FLOOR = 38, FGT_OP_CEIL = 39,
  FGT_OP_ROUND = 40, FGT_OP_BITWISE_NOT = 41,
  /* predicates */
  FGT_OP_COMPARE = 50,        /* predicate field; result bool                          */
  FGT_OP_SELECT = 51,         /* (bool cond, a, b)                                     */
  /* reductions: attrs = sorted reduced axes (argmax/argmin: attrs[0] = axis) */
  FGT_OP_REDUCE_SUM = 60, FGT_OP_REDUCE_MAX = 61, FGT_OP_REDUCE_MIN = 62,
  FGT_OP_REDUCE_PROD = 63, FGT_OP_REDUCE_ANY = 64, FGT_OP_REDUCE_ALL = 65,
  FGT_OP_ARGMAX = 66, FGT_OP_ARGMIN = 67,
  /* index transforms (src/fugatensor/lowering.py:103-111, ir/tensor_rules.py:124-237) */
  FGT_OP_SLICE = 70,          /* attrs = starts[rank], steps[rank]; stops follow from  */
                              /* the result shape                                      */
  FGT_OP_PAD = 71,            /* (x, pad value: rank 0, same dtype); attrs = low[rank], */
                              /* interior[rank]; high follows from the result shape    */
  FGT_OP_CONCATENATE = 72,    /* two operands joined along attrs[0] (longer lists nest) */
  FGT_OP_GATHER = 73,         /* (params, indices i32/i64); attrs[0] = axis; indices    */
                              /* outside [0, extent) read 0                            */
  FGT_OP_SCATTER_ADD = 74     /* (base, indices, updates); attrs[0] = axis; result =    */
                              /* base plus updates at indices (outside: dropped)       */
} fgt_opcode;

typedef enum fgt_predicate {
  FGT_CMP_EQ = 0, FGT_CMP_NE = 1, FGT_CMP_LT = 2, FGT_CMP_LE = 3, FGT_CMP_GT = 4, FGT_CMP_GE = 5
} fgt_predicate;

/* One SSA value. Operands refer to earlier nodes (topological order). The
 * declared dtype/shape must equal what Fuga's typing rule infers. */
typedef struct fgt_node {
  int32_t opcode;
  int32_t dtype;
  int32_t rank;
  int32_t num_operands;
  int64_t shape[FGT_MAX_RANK];
  int32_t operands[FGT_MAX_OPERANDS];
  int32_t num_attrs;
  int64_t attrs[FGT_MAX_ATTRS];
  int32_t predicate;
  int32_t reserved;
  uint64_t constant_bits;
} fgt_node;

typedef struct fgt_partition_desc {
  int32_t abi_version;        /* FGT_ABI_VERSION                                       */
  int32_t num_nodes;
  const fgt_node* nodes;
  int32_t num_outputs;
  const int32_t* outputs;     /* node ids, in output-port order (repeats allowed)      */
} fgt_partition_desc;

/* How floating reductions accumulate. */
typedef enum fgt_accumulation {
  /* f16/bf16 sums accumulate in f32 and f32 sums in f32 spans folded into f64;
   * the result is rounded once to the reduction's dtype (default). */
  FGT_ACCUM_WIDE = 0,
  /* every partial sum is rounded to the reduction's dtype, as the reference's
   * storage-dtype reductions do (tests/test_tensor_primitives.py:184-192). */
  FGT_ACCUM_STORAGE = 1
} fgt_accumulation;

typedef struct fgt_spec_options {
  int32_t accumulation;       /* fgt_accumulation                                      */
  int32_t shard_world;        /* 0/1 = unsharded; N>1 = leading-dim shard over N ranks */
  int32_t shard_rank;
  int32_t row_elems;          /* block-per-row kernels: elements per thread per row    */
                              /* operand (0: the library's choice)                     */
  uint64_t shard_inputs;      /* bit i set: input port i is split along dim 0          */
  const char* cache_dir;      /* compiled-kernel disk cache (NULL: FGT_CACHE_DIR env)  */
  int32_t ring_kb;            /* row kernels: shared-memory row ring budget per CTA in */
                              /* KB (0: the library's choice, 96)                      */
  int32_t row_cluster;        /* block-per-row kernels: CTAs of a thread-block cluster */
                              /* sharing each row (0/1: none; 2, 4, 8)                 */
  int32_t row_flags;          /* block-per-row kernels, fgt_row_flag bits (0: none)    */
} fgt_spec_options;

typedef enum fgt_row_flag {
  /* a kernel whose registers are within reach of one more resident CTA per SM
   * is compiled bounded to that many (kept when it spills at most 256 bytes) */
  FGT_ROW_OCCUPANCY_STEP = 1,
  /* exp computed by CUDA's expf everywhere, instead of the library's exp
   * (2^f by ex2.approx, 2^n in the exponent field) in redoable row phases */
  FGT_ROW_EXPF = 2,
  /* column-reduction accumulators in shared memory (one private slot per
   * thread and element) instead of registers */
  FGT_ROW_SMEM_COLS = 4,
  /* cross-warp row reductions by a shuffle butterfly over the warp partials,
   * instead of every thread folding them from shared memory */
  FGT_ROW_XW_SHUFFLE = 8,
  /* row operands stay in the shared-memory ring while their row is computed
   * (each phase reads the thread's own pieces again), and per-thread column
   * operands of 16-bit types stay packed two per register: fewer registers
   * per thread, so more CTAs per SM, for rows with several phases */
  FGT_ROW_RING_RESIDENT = 16,
  /* every phase after a row's first reads the row operands (and per-thread
   * column operands) through copies the compiler cannot see through, so each
   * phase recomputes its element values instead of the compiler keeping the
   * earlier phases' values live: fewer registers for rows with several
   * phases, at the price of recomputation */
  FGT_ROW_PHASE_COPIES = 32,
  /* per-thread column operands of 16-bit types (gamma) held two per 32-bit
   * register, as in FGT_ROW_RING_RESIDENT, without keeping rows in the ring */
  FGT_ROW_PACK_COLS = 64,
  /* column-reduction accumulators (dgamma, dbeta) in the SM's tensor memory
   * (tcgen05.alloc / ld / st): each thread keeps its columns in its own TMEM
   * lane and reads and writes one chunk at a time, so they hold neither
   * registers nor shared memory; f32 sums over block-per-row kernels of a
   * multiple of 128 threads only (others keep registers) */
  FGT_ROW_TMEM_COLS = 128,
  /* in partitions whose floating outputs are all f16 / bf16, element
   * divisions by a row constant d are computed as x * RN(1/d) (at most one
   * ulp of f32 from the IEEE quotient, which the 16-bit rounding of the
   * outputs hides but for rounding ties), without the per-element range
   * checks of the exact form; a row whose divisor has no normal reciprocal
   * is computed with IEEE division. Other partitions are unchanged. */
  FGT_ROW_NARROW_DIV = 256
} fgt_row_flag;

typedef struct fgt_spec fgt_spec;   /* opaque: planned + compiled partition       */
typedef struct fgt_comm fgt_comm;   /* opaque: one rank of an NCCL communicator   */

typedef struct fgt_spec_info {
  int32_t num_inputs;
  int32_t num_outputs;
  int32_t kernel_count;       /* launches per fgt_spec_launch (collectives excluded)  */
  int32_t collective_count;   /* NCCL calls per sharded launch                        */
  size_t workspace_bytes;     /* scratch the caller must pass (256-byte aligned)      */
} fgt_spec_info;

/* Last error message of the calling thread (never NULL). */
const char* fgt_last_error(void);

/* ABI version of the loaded library. */
int32_t fgt_abi_version(void);

/* Type-check, plan, specialise and compile a partition.
 * Replaces the CUDA branch of Engine._compile (src/fugatensor/engine.py:344-353):
 * ASK partition (cpp/compiler.cpp:44-48, src/fugatensor/_ask/gpu.py:71) and the
 * owned-step LLVM->cubin build (src/fugatensor/_ask/gpu.py:160-216,
 * src/fugatensor/_ask/cuda.py:185-313). options may be NULL. */
fgt_status fgt_spec_create(const fgt_partition_desc* desc, const fgt_spec_options* options,
                           fgt_spec** out);

void fgt_spec_destroy(fgt_spec* spec);

fgt_status fgt_spec_get_info(const fgt_spec* spec, fgt_spec_info* info);

/* Shape/dtype of an input or output port (is_output 0/1). */
fgt_status fgt_spec_port(const fgt_spec* spec, int32_t is_output, int32_t index,
                         int32_t* dtype, int32_t* rank, int64_t* shape);

/* Execution Plan v1 JSON (src/fugatensor/_ask/plan.py:21-86) of the launch plan,
 * plus a cuda_lowering report. Copies at most capacity bytes (NUL-terminated);
 * *needed receives the full length + 1. */
fgt_status fgt_spec_plan_json(const fgt_spec* spec, char* buffer, size_t capacity, size_t* needed);

/* Generated CUDA source of kernel `index` (diagnostics; same copy contract). */
fgt_status fgt_spec_kernel_source(const fgt_spec* spec, int32_t index, char* buffer,
                                  size_t capacity, size_t* needed);

/* Launch every kernel of the partition on `stream` (a cudaStream_t/CUstream,
 * NULL = legacy default stream), in stream order, asynchronously.
 * Replaces ProgramPorts::runFastCore -> PreparedProgram::run
 * (cpp/ask_runtime.cpp:412-463) and the cache-hit dispatch at
 * cpp/lazy.cpp:946-948. inputs/outputs are device pointers in port order;
 * workspace must hold fgt_spec_info.workspace_bytes (may be NULL when 0).
 * Outputs may alias each other when the partition repeats a node; they must
 * not overlap inputs. Capturable in a CUDA graph. */
fgt_status fgt_spec_launch(const fgt_spec* spec, const void* const* inputs, void* const* outputs,
                           void* workspace, size_t workspace_bytes, void* stream);

/* ---- prepared programs: CUDA graph replay ------------------------------- */

typedef struct fgt_program fgt_program;  /* opaque: a spec prepared for replay */

/* Prepare `spec` for repeated runs. With use_graph != 0 the first run on a
 * CUDA context instantiates the spec's kernels as one CUDA graph (a chain of
 * kernel nodes); every later run writes its buffers into the graph's kernel
 * nodes and replays it with one cuGraphLaunch. use_graph = 0 launches the
 * kernels one by one, as fgt_spec_launch. Replaces
 * PreparedCUDAProgram(..., graph=True) -> prepare_program
 * (src/fugatensor/_ask/executable.py:120-152, cpp/ask_runtime.cpp:789-843)
 * and its cached dispatch ProgramPorts::runFastCore
 * (cpp/ask_runtime.cpp:412-463, called at cpp/lazy.cpp:946-948).
 * The spec must outlive the program. Specs that reduce over a sharded
 * dimension (collectives) are rejected with FGT_ERR_UNSUPPORTED. */
fgt_status fgt_program_create(const fgt_spec* spec, int32_t use_graph, fgt_program** out);

/* Run the program on `stream`: same buffer contract and validation as
 * fgt_spec_launch (checked before anything is enqueued). Runs of one
 * program from several threads are serialised on the program's lock. The
 * first graph run on a context instantiates the graph (host and driver
 * resources). On a stream that is being captured the kernels are launched
 * one by one instead, so they become nodes of the caller's graph. */
fgt_status fgt_program_run(fgt_program* program, const void* const* inputs, void* const* outputs, void* workspace,
                           size_t workspace_bytes, void* stream);

/* Kernels one run launches (graph nodes). */
int32_t fgt_program_kernel_count(const fgt_program* program);

void fgt_program_destroy(fgt_program* program);

/* ---- leading-dimension sharding across GPUs (one process per GPU) ------- */

/* 128-byte NCCL unique id, created on one rank and shared by the caller. */
fgt_status fgt_comm_unique_id(uint8_t id[128]);

/* Join a communicator of `world` ranks on the current device. No reference
 * counterpart: the reference binds one Engine to one device
 * (src/fugatensor/engine.py:145,237-239). The communicator is non-blocking:
 * initialisation and every later collective enqueue are polled against a
 * deadline of FGT_COMM_TIMEOUT_MS milliseconds (environment, default 300000).
 * A rank that never joins, or an NCCL error, ends in FGT_ERR_NCCL and the
 * communicator is aborted; a sharded launch on an aborted or failed
 * communicator returns FGT_ERR_NCCL before launching any kernel.
 * With world > 1 (up to 8 ranks on one machine) every rank also allocates a
 * peer mailbox (16 MiB + 64 KiB of device memory) and maps every other
 * rank's through CUDA IPC; reductions over the sharded dimension then
 * exchange their per-rank records inside one finalising kernel with NVLink
 * stores and flags, instead of an NCCL all-gather between two kernels. The
 * ranks decide together; if any rank cannot map the mailboxes, or
 * FGT_PEER_EXCHANGE=0, all use the NCCL path. A kernel waits at most
 * FGT_EXCHANGE_WAIT_MS (default 10000) for a peer's record; on a timeout it
 * marks the communicator and the next sharded launch returns FGT_ERR_NCCL.
 * Launches on one communicator must not overlap on the GPU (as for NCCL). */
fgt_status fgt_comm_create(const uint8_t id[128], int32_t world, int32_t rank, fgt_comm** out);

/* 1 when the communicator exchanges records through peer mailboxes, 0 when
 * through NCCL. */
int32_t fgt_comm_peer_exchange(const fgt_comm* comm);

/* Collective when the communicator has peer mailboxes: every rank calls it
 * after its last launch; no rank unmaps its mailbox before all have met. */
void fgt_comm_destroy(fgt_comm* comm);

/* Sharded launch of a spec created with options.shard_world == world of comm.
 * inputs flagged in shard_inputs hold this rank's contiguous dim-0 slab; other
 * inputs are replicated. Row-local outputs are this rank's slab; outputs that
 * reduce over the sharded dimension are combined across ranks (NCCL
 * all-gather of per-rank partials + an ordered on-device combine) and are
 * replicated, identical on every rank. */
fgt_status fgt_spec_launch_sharded(const fgt_spec* spec, fgt_comm* comm, const void* const* inputs,
                                   void* const* outputs, void* workspace, size_t workspace_bytes,
                                   void* stream);

/* ---- allocation-free whole-tensor reduction ----------------------------- */

/* Scratch limits of fgt_reduce_f32_noalloc. */
#define FGT_NOALLOC_SLOTS 2048
#define FGT_NOALLOC_ELEMS_PER_SLOT (1LL << 20)
#define FGT_NOALLOC_SCRATCH_BYTES (FGT_NOALLOC_SLOTS * 32)

/* No counterpart in the reference: for callers that cannot allocate device
 * memory (code running inside an allocator or memory manager, services that
 * must not touch the device allocator after start-up, hosts that own all
 * device memory and pass only input/output buffers). Computes the sum, IEEE
 * max, first-occurrence argmax (NaN counts as the maximum) and mean (sum / n)
 * of x[0..n), like the whole-tensor reduction partition through
 * fgt_spec_launch (every element added into an f64 accumulator, the total
 * rounded to f32 once), but keeps its per-CTA partials in a static 64 KiB
 * device array instead of a caller workspace. It calls no cudaMalloc,
 * cudaFree or allocating library routine.
 *   - x: device pointer, 16-byte aligned; sum/max/mean: device f32 scalars;
 *     argmax: device i64 scalar; stream: cudaStream_t (NULL = default).
 *   - n must be in [1, 2^31] (FGT_NOALLOC_SLOTS x FGT_NOALLOC_ELEMS_PER_SLOT);
 *     larger n is rejected with FGT_ERR_INVALID before any launch.
 *   - The array is loaded on every GPU that uses the library and stays until
 *     exit. All calls on a device share it: calls that overlap on the GPU
 *     race. Nothing in it needs to start at zero (each call writes every slot
 *     it reads).
 *   - Set-up: the first call on a device (and in each new CUDA context of it,
 *     e.g. after cudaDeviceReset) looks up the array's device address with
 *     cudaGetSymbolAddress. Under CUDA's lazy module loading (the default
 *     since 12.2) that lookup is when the driver loads the library's module
 *     and commits the array's device memory. So make the first call on each
 *     device at start-up (a call on a small valid input will do), outside any
 *     allocator hook and before any stream capture; later calls touch no
 *     device memory beyond their inputs, outputs and the array.
 *   - A CUDA error already pending on the calling thread is reported (and left
 *     pending) without launching. */
fgt_status fgt_reduce_f32_noalloc(const float* x, int64_t n, float* sum, float* max, int64_t* argmax, float* mean,
                                  void* stream);

#ifdef __cplusplus
}
#endif
#endif /* FGT_H_ */
