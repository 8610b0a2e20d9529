// fgt_noalloc.cu — whole-tensor f32 sum / max / argmax / mean without any
// allocation, for callers that cannot call cudaMalloc: code running where
// allocation is forbidden or unavailable (inside a custom memory manager or
// allocator callback, a real-time or pre-reserved-memory service that must
// not touch the device allocator after start-up, or a host framework that
// owns all device memory and hands out only input/output buffers).
//
// It computes the same results as the whole-tensor reduction partition
// (sum, amax, argmax, mean of one f32 array) launched through
// fgt_spec_launch: every element is added into an f64 accumulator and the
// total is rounded to f32 once (so exactly cancelling terms sum to the exact
// result, as in the generated kernel), IEEE max
// (NaN propagates, +0 beats -0), first-occurrence argmax with NaN counted as
// the maximum, mean = sum / n with one IEEE division. The difference is where
// the scratch lives: the per-CTA partials are kept in a file-scope device
// array instead of a caller-provided workspace.
//
// Limits and rules (stated again in include/fgt.h):
//   - the scratch array holds FGT_NOALLOC_SLOTS partial records; each slot
//     covers FGT_NOALLOC_ELEMS_PER_SLOT elements, so n is limited to
//     FGT_NOALLOC_SLOTS * FGT_NOALLOC_ELEMS_PER_SLOT = 2^31 elements; larger n
//     is rejected with FGT_ERR_INVALID before anything is launched;
//   - every GPU that loads the library holds the array (64 KiB) until exit;
//   - all calls on a device share the array: calls that overlap on the GPU
//     (different streams, or graphs replayed concurrently) race on it;
//   - set-up: the first call on a device looks up the array's device address
//     with cudaGetSymbolAddress (once per device and CUDA context, under a
//     lock). With CUDA's lazy module loading (the default since 12.2) that
//     first lookup is also when the driver loads this module and commits the
//     64 KiB array, so the first call on each device is the one that touches
//     device memory: make it at start-up, outside any allocator hook and
//     before any stream capture. If the context is destroyed and re-created
//     (cudaDeviceReset), the next call sees a new context id and repeats the
//     set-up;
//   - nothing in the array needs to start at zero: every slot the finalising
//     kernel reads is written earlier in the same call.
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "fgt.h"
#include "fgt_device.cuh"
#include "fgt_driver.h"

namespace fgt {
fgt_status record_error(fgt_status s, const std::string& m);  // fgt_runtime.cpp
}

namespace {

constexpr int kThreads = 256;
constexpr int kVec = 4;
constexpr long long kElemsPerSlot = 1ll << 20;

struct Slot {            // one CTA's partial record (32 bytes)
  double sum;
  float max;
  float amax_val;
  long long amax_idx;
  long long pad_;
};
static_assert(sizeof(Slot) == 32, "slot layout");
static_assert(FGT_NOALLOC_SLOTS * sizeof(Slot) == FGT_NOALLOC_SCRATCH_BYTES, "scratch size");
static_assert(kElemsPerSlot == FGT_NOALLOC_ELEMS_PER_SLOT, "slot span");

static __device__ __align__(256) unsigned char fgt_noalloc_scratch[FGT_NOALLOC_SCRATCH_BYTES];

// Block combine of (sum, max, argmax) in warp order; every thread ends with
// the block's values (the same deterministic order as the generated kernels).
__device__ void block_combine(double& sum, float& mx, float& av, long long& ai) {
  __shared__ double s_sum[kThreads / 32];
  __shared__ float s_max[kThreads / 32], s_av[kThreads / 32];
  __shared__ long long s_ai[kThreads / 32];
#pragma unroll
  for (int m = 1; m < 32; m <<= 1) {
    sum += fgt_shfl_xor(sum, m);
    mx = fgt_fmax(mx, fgt_shfl_xor(mx, m));
    const float ov = fgt_shfl_xor(av, m);
    const long long oi = fgt_shfl_xor((fgt_i64)ai, m);
    if (fgt_arg_better_f<true>(ov, oi, av, ai)) {
      av = ov;
      ai = oi;
    }
  }
  const int w = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) {
    s_sum[w] = sum;
    s_max[w] = mx;
    s_av[w] = av;
    s_ai[w] = ai;
  }
  __syncthreads();
  sum = s_sum[0];
  mx = s_max[0];
  av = s_av[0];
  ai = s_ai[0];
  for (int k = 1; k < kThreads / 32; ++k) {
    sum += s_sum[k];
    mx = fgt_fmax(mx, s_max[k]);
    if (fgt_arg_better_f<true>(s_av[k], s_ai[k], av, ai)) {
      av = s_av[k];
      ai = s_ai[k];
    }
  }
  __syncthreads();
}

// One CTA per slot: elements [slot * kElemsPerSlot, min(n, (slot+1) * kElemsPerSlot)).
__global__ void __launch_bounds__(kThreads) noalloc_partials(const float* __restrict__ x, long long n, Slot* slots) {
  const long long lo = (long long)blockIdx.x * kElemsPerSlot;
  const long long hi = lo + kElemsPerSlot < n ? lo + kElemsPerSlot : n;
  double sum = 0.0;
  float mx = __int_as_float(0xff800000);
  float av = __int_as_float(0xff800000);
  long long ai = 9223372036854775807ll;
  // full vectors (the caller's x is 16-byte aligned; slot bounds are multiples of 4)
  const long long vhi = lo + ((hi - lo) / kVec) * kVec;
  for (long long e0 = lo + (long long)threadIdx.x * kVec; e0 < vhi; e0 += (long long)kThreads * kVec) {
    float v[kVec];
    fgt_vload(v, x + e0);
    float lm = v[0], la = v[0];
    int li = 0;
#pragma unroll
    for (int k = 0; k < kVec; ++k) {
      sum += (double)v[k];  // each element into the f64 lane: the total rounds once, at the end
      lm = fgt_fmax(lm, v[k]);
      if (k && fgt_arg_scan_f<true>(v[k], la, li, 0x7fffffff)) {
        la = v[k];
        li = k;
      }
    }
    mx = fgt_fmax(mx, lm);
    const long long gi = e0 + li;
    if (fgt_arg_scan_f<true>(la, av, ai, 9223372036854775807ll)) {
      av = la;
      ai = gi;
    }
  }
  for (long long e = vhi + threadIdx.x; e < hi; e += kThreads) {  // tail (< 4 elements)
    const float v = x[e];
    sum += (double)v;
    mx = fgt_fmax(mx, v);
    if (fgt_arg_scan_f<true>(v, av, ai, 9223372036854775807ll)) {
      av = v;
      ai = e;
    }
  }
  block_combine(sum, mx, av, ai);
  if (threadIdx.x == 0) {
    Slot s;
    s.sum = sum;
    s.max = mx;
    s.amax_val = av;
    s.amax_idx = ai;
    s.pad_ = 0;
    slots[blockIdx.x] = s;
  }
}

__global__ void __launch_bounds__(kThreads) noalloc_finalize(const Slot* slots, int nslots, long long n, float* sum_out,
                                                             float* max_out, long long* argmax_out, float* mean_out) {
  double sum = 0.0;
  float mx = __int_as_float(0xff800000);
  float av = __int_as_float(0xff800000);
  long long ai = 9223372036854775807ll;
  for (int k = threadIdx.x; k < nslots; k += kThreads) {
    const Slot s = slots[k];
    sum += s.sum;
    mx = fgt_fmax(mx, s.max);
    if (fgt_arg_better_f<true>(s.amax_val, s.amax_idx, av, ai)) {
      av = s.amax_val;
      ai = s.amax_idx;
    }
  }
  block_combine(sum, mx, av, ai);
  if (threadIdx.x == 0) {
    const float s32 = __double2float_rn(sum);
    *sum_out = s32;
    *max_out = mx;
    *argmax_out = ai;
    *mean_out = __fdiv_rn(s32, (float)n);
  }
}

// Set-up state per device ordinal: the array's device address in the CUDA
// context it was looked up in (identified by the driver's process-unique
// context id, or by the context handle on a driver without cuCtxGetId).
struct Setup {
  void* addr = nullptr;
  unsigned long long ctx_id = 0;
};
std::mutex g_setup_mu;
Setup g_setup[64];

bool current_context_id(unsigned long long* id) {
  fgt::Driver& d = fgt::drv();
  if (!d.ok) return false;
  CUcontext ctx = nullptr;
  if (d.CtxGetCurrent(&ctx) != CUDA_SUCCESS || !ctx) return false;
  if (d.CtxGetId) return d.CtxGetId(ctx, id) == CUDA_SUCCESS;
  *id = (unsigned long long)(uintptr_t)ctx;
  return true;
}

// Failures are reported like every other entry point: status code plus the
// thread's fgt_last_error() message.
fgt_status fail(fgt_status s, const std::string& m) { return fgt::record_error(s, m); }

}  // namespace

extern "C" fgt_status fgt_reduce_f32_noalloc(const float* x, int64_t n, float* sum, float* max, int64_t* argmax,
                                             float* mean, void* stream) {
  if (n <= 0) return fail(FGT_ERR_INVALID, "fgt_reduce_f32_noalloc: n must be positive (argmax of an empty array)");
  if (n > (int64_t)FGT_NOALLOC_SLOTS * FGT_NOALLOC_ELEMS_PER_SLOT)
    return fail(FGT_ERR_INVALID, "fgt_reduce_f32_noalloc: n = " + std::to_string(n) +
                                     " exceeds the static scratch limit of 2^31 elements (" +
                                     std::to_string(FGT_NOALLOC_SLOTS) + " slots x 2^20 elements)");
  if (!x || !sum || !max || !argmax || !mean) return fail(FGT_ERR_INVALID, "fgt_reduce_f32_noalloc: NULL buffer");
  if ((uintptr_t)x % 16) return fail(FGT_ERR_INVALID, "fgt_reduce_f32_noalloc: x must be 16-byte aligned");
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(FGT_ERR_CUDA, std::string("cudaGetDevice: ") + cudaGetErrorString(e));
  if (dev < 0 || dev >= 64) return fail(FGT_ERR_CUDA, "fgt_reduce_f32_noalloc: device ordinal out of range");
  // An error left pending by earlier, unrelated CUDA work on this thread is
  // reported as such (and left pending), not blamed on this call's launches.
  e = cudaPeekAtLastError();
  if (e != cudaSuccess)
    return fail(FGT_ERR_CUDA, std::string("fgt_reduce_f32_noalloc: an earlier CUDA error is pending on this thread (") +
                                  cudaGetErrorString(e) + "); nothing was launched");
  void* scratch = nullptr;
  {
    // Set-up, once per device and context, with that device current: the
    // array's device address. Host code only ever passes this address to the
    // kernels, never the symbol (a host-side stand-in).
    std::lock_guard<std::mutex> lock(g_setup_mu);
    Setup& su = g_setup[dev];
    unsigned long long id = 0;
    const bool have_id = current_context_id(&id);
    if (!su.addr || !have_id || id != su.ctx_id) {
      void* p = nullptr;
      e = cudaGetSymbolAddress(&p, fgt_noalloc_scratch);
      if (e != cudaSuccess) return fail(FGT_ERR_CUDA, std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(e));
      // the lookup made the device's context current if none was
      if (!current_context_id(&id)) return fail(FGT_ERR_CUDA, "fgt_reduce_f32_noalloc: no current CUDA context");
      su.addr = p;
      su.ctx_id = id;
    }
    scratch = su.addr;
  }
  const int nslots = (int)((n + FGT_NOALLOC_ELEMS_PER_SLOT - 1) / FGT_NOALLOC_ELEMS_PER_SLOT);
  cudaStream_t st = (cudaStream_t)stream;
  Slot* slots = static_cast<Slot*>(scratch);
  noalloc_partials<<<nslots, kThreads, 0, st>>>(x, (long long)n, slots);
  e = cudaGetLastError();
  if (e != cudaSuccess) return fail(FGT_ERR_CUDA, std::string("launch (partials): ") + cudaGetErrorString(e));
  noalloc_finalize<<<1, kThreads, 0, st>>>(slots, nslots, (long long)n, sum, max, (long long*)argmax, mean);
  e = cudaGetLastError();
  if (e != cudaSuccess) return fail(FGT_ERR_CUDA, std::string("launch (finalize): ") + cudaGetErrorString(e));
  return FGT_OK;
}
