// fgt_runtime.cpp — the C ABI: spec creation (plan + specialise + compile),
// launch on a caller stream, and leading-dimension sharded launches.
//
// Replaces, for the fused elementwise / reduction partitions, the reference's
//   - owned-step build: ASK emit_cuda_llvm -> llc -> ptxas
//     (src/fugatensor/_ask/gpu.py:160-216, src/fugatensor/_ask/cuda.py:185-313)
//     here: template specialisation -> NVRTC (sm_100a, -fmad=false) -> cubin,
//     cached on disk by content hash like the reference's IR/cubin caches
//     (src/fugatensor/_ask/cache.py);
//   - PreparedProgram::run / ProgramPorts::runFastCore
//     (cpp/ask_runtime.cpp:412-463): stream-ordered cuLaunchKernel of the
//     plan's kernels with caller-owned buffers and workspace.
#include <nvrtc.h>

#include <cctype>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <memory>
#include <mutex>
#include <algorithm>
#include <climits>
#include <thread>
#include <chrono>
#include <sstream>
#include <dlfcn.h>
#include <sys/stat.h>
#include <unistd.h>

#include "fgt_driver.h"
#include "fgt_plan.h"

extern const char* const fgt_device_library_source;  // fgt_device.cuh, embedded at build time

namespace fgt {
namespace {

thread_local std::string g_last_error = "";

fgt_status set_error(fgt_status s, const std::string& m) {
  g_last_error = m;
  return s;
}

void cu_check(CUresult r, const char* what) {
  if (r != CUDA_SUCCESS) {
    const char* name = nullptr;
    const char* msg = nullptr;
    drv().GetErrorName(r, &name);
    drv().GetErrorString(r, &msg);
    fail(FGT_ERR_CUDA, std::string(what) + ": " + (name ? name : "?") + " (" + (msg ? msg : "") + ")");
  }
}

uint64_t fnv1a(const std::string& s, uint64_t h = 1469598103934665603ULL) {
  for (unsigned char c : s) {
    h ^= c;
    h *= 1099511628211ULL;
  }
  return h;
}

std::string cache_root(const char* opt_dir) {
  if (opt_dir && *opt_dir) return opt_dir;
  const char* env = std::getenv("FGT_CACHE_DIR");
  if (env && *env) return env;
  const char* home = std::getenv("HOME");
  return std::string(home ? home : "/tmp") + "/.cache/fgt_b200";
}

void mkdirs(const std::string& path) {
  std::string cur;
  for (size_t i = 0; i < path.size(); ++i) {
    cur += path[i];
    if (path[i] == '/' && i > 0) mkdir(cur.c_str(), 0755);
  }
  mkdir(path.c_str(), 0755);
}

const char* kNvrtcOptions[] = {"-arch=sm_100a", "-fmad=false", "-std=c++17", "-default-device", "-lineinfo",
                               "-prec-div=true", "-prec-sqrt=true", "-ftz=false", "-Xptxas=-v"};

struct Compiled {
  std::string cubin;
  int regs = -1, spill_bytes = -1;  // from ptxas's verbose report (-1: not reported)
};

// ptxas -v reports "Used N registers" and "N bytes spill stores".
void parse_ptxas_report(const std::string& log, Compiled* c) {
  size_t p = log.find("Used ");
  int v = 0;
  if (p != std::string::npos && std::sscanf(log.c_str() + p, "Used %d registers", &v) == 1) c->regs = v;
  p = log.find(" bytes spill stores");
  if (p != std::string::npos) {
    size_t b = p;
    while (b > 0 && std::isdigit((unsigned char)log[b - 1])) --b;
    if (b < p) c->spill_bytes = std::atoi(log.c_str() + b);
  }
}

// SHA-256 (FIPS 180-4) of a byte string, as 64 hex digits: the content check
// stored beside each cached cubin (its file name carries a 64-bit FNV-1a hash).
std::string sha256_hex(const std::string& msg) {
  static const uint32_t K[64] = {
      0x428a2f98, 0x71374491, 0xb5c0fbcf, 0xe9b5dba5, 0x3956c25b, 0x59f111f1, 0x923f82a4, 0xab1c5ed5, 0xd807aa98, 0x12835b01,
      0x243185be, 0x550c7dc3, 0x72be5d74, 0x80deb1fe, 0x9bdc06a7, 0xc19bf174, 0xe49b69c1, 0xefbe4786, 0x0fc19dc6, 0x240ca1cc,
      0x2de92c6f, 0x4a7484aa, 0x5cb0a9dc, 0x76f988da, 0x983e5152, 0xa831c66d, 0xb00327c8, 0xbf597fc7, 0xc6e00bf3, 0xd5a79147,
      0x06ca6351, 0x14292967, 0x27b70a85, 0x2e1b2138, 0x4d2c6dfc, 0x53380d13, 0x650a7354, 0x766a0abb, 0x81c2c92e, 0x92722c85,
      0xa2bfe8a1, 0xa81a664b, 0xc24b8b70, 0xc76c51a3, 0xd192e819, 0xd6990624, 0xf40e3585, 0x106aa070, 0x19a4c116, 0x1e376c08,
      0x2748774c, 0x34b0bcb5, 0x391c0cb3, 0x4ed8aa4a, 0x5b9cca4f, 0x682e6ff3, 0x748f82ee, 0x78a5636f, 0x84c87814, 0x8cc70208,
      0x90befffa, 0xa4506ceb, 0xbef9a3f7, 0xc67178f2};
  uint32_t h[8] = {0x6a09e667, 0xbb67ae85, 0x3c6ef372, 0xa54ff53a, 0x510e527f, 0x9b05688c, 0x1f83d9ab, 0x5be0cd19};
  auto rotr = [](uint32_t x, int n) { return (x >> n) | (x << (32 - n)); };
  std::string m = msg;
  const uint64_t bits = (uint64_t)msg.size() * 8;
  m.push_back((char)0x80);
  while (m.size() % 64 != 56) m.push_back(0);
  for (int i = 7; i >= 0; --i) m.push_back((char)((bits >> (8 * i)) & 0xff));
  for (size_t off = 0; off < m.size(); off += 64) {
    uint32_t w[64];
    for (int i = 0; i < 16; ++i) {
      const unsigned char* b = (const unsigned char*)m.data() + off + 4 * i;
      w[i] = ((uint32_t)b[0] << 24) | ((uint32_t)b[1] << 16) | ((uint32_t)b[2] << 8) | b[3];
    }
    for (int i = 16; i < 64; ++i) {
      const uint32_t s0 = rotr(w[i - 15], 7) ^ rotr(w[i - 15], 18) ^ (w[i - 15] >> 3);
      const uint32_t s1 = rotr(w[i - 2], 17) ^ rotr(w[i - 2], 19) ^ (w[i - 2] >> 10);
      w[i] = w[i - 16] + s0 + w[i - 7] + s1;
    }
    uint32_t a = h[0], b = h[1], c = h[2], d = h[3], e = h[4], f = h[5], g = h[6], hh = h[7];
    for (int i = 0; i < 64; ++i) {
      const uint32_t S1 = rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25);
      const uint32_t ch = (e & f) ^ (~e & g);
      const uint32_t t1 = hh + S1 + ch + K[i] + w[i];
      const uint32_t S0 = rotr(a, 2) ^ rotr(a, 13) ^ rotr(a, 22);
      const uint32_t mj = (a & b) ^ (a & c) ^ (b & c);
      const uint32_t t2 = S0 + mj;
      hh = g;
      g = f;
      f = e;
      e = d + t1;
      d = c;
      c = b;
      b = a;
      a = t1 + t2;
    }
    h[0] += a, h[1] += b, h[2] += c, h[3] += d, h[4] += e, h[5] += f, h[6] += g, h[7] += hh;
  }
  char out[65];
  for (int i = 0; i < 8; ++i) std::snprintf(out + 8 * i, 9, "%08x", h[i]);
  return std::string(out, 64);
}

std::string read_file(const std::string& path) {
  std::ifstream f(path, std::ios::binary);
  if (!f) return std::string();
  std::stringstream ss;
  ss << f.rdbuf();
  return ss.str();
}

// Atomic publish: write a private file, then rename.
void publish(const std::string& path, const std::string& data) {
  const std::string tmp = path + ".tmp." + std::to_string(getpid());
  {
    std::ofstream f(tmp, std::ios::binary);
    f.write(data.data(), (std::streamsize)data.size());
  }
  std::rename(tmp.c_str(), path.c_str());
}

// NVRTC compile of one kernel, cached on disk by a hash of the compiler
// version, options and source. The ptxas register report is cached beside
// the cubin (".regs": "<registers> <spill bytes>"), and so is the SHA-256 of
// the full key (".key"): a cached cubin is used only when that digest
// matches, and a 64-bit name collision moves on to the next slot (-1, -2, ...).
// NVRTC, opened at run time. The toolkit's library (the CUDA the library was
// built with, FGT_CUDA_LIB_DIR) comes first, by its full path: a process that
// imported PyTorch already holds PyTorch's own, older libnvrtc.so.12, and a
// plain soname lookup would bind that one. FGT_NVRTC names another library.
struct NvrtcApi {
  nvrtcResult (*Version)(int*, int*) = nullptr;
  nvrtcResult (*CreateProgram)(nvrtcProgram*, const char*, const char*, int, const char* const*, const char* const*) = nullptr;
  nvrtcResult (*CompileProgram)(nvrtcProgram, int, const char* const*) = nullptr;
  nvrtcResult (*GetProgramLogSize)(nvrtcProgram, size_t*) = nullptr;
  nvrtcResult (*GetProgramLog)(nvrtcProgram, char*) = nullptr;
  nvrtcResult (*GetCUBINSize)(nvrtcProgram, size_t*) = nullptr;
  nvrtcResult (*GetCUBIN)(nvrtcProgram, char*) = nullptr;
  nvrtcResult (*DestroyProgram)(nvrtcProgram*) = nullptr;
  std::string path;
};

#ifndef FGT_CUDA_LIB_DIR
#define FGT_CUDA_LIB_DIR "/usr/local/cuda/lib64"
#endif

const NvrtcApi& nvrtc() {
  static NvrtcApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    std::vector<std::string> names;
    if (const char* e = std::getenv("FGT_NVRTC")) names.push_back(e);
    names.push_back(std::string(FGT_CUDA_LIB_DIR) + "/libnvrtc.so.12");
    names.push_back("libnvrtc.so.12");
    for (const std::string& n : names) {
      void* h = dlopen(n.c_str(), RTLD_NOW | RTLD_LOCAL);
      if (!h) continue;
      auto sym = [&](const char* s) { return dlsym(h, s); };
      api.Version = (decltype(api.Version))sym("nvrtcVersion");
      api.CreateProgram = (decltype(api.CreateProgram))sym("nvrtcCreateProgram");
      api.CompileProgram = (decltype(api.CompileProgram))sym("nvrtcCompileProgram");
      api.GetProgramLogSize = (decltype(api.GetProgramLogSize))sym("nvrtcGetProgramLogSize");
      api.GetProgramLog = (decltype(api.GetProgramLog))sym("nvrtcGetProgramLog");
      api.GetCUBINSize = (decltype(api.GetCUBINSize))sym("nvrtcGetCUBINSize");
      api.GetCUBIN = (decltype(api.GetCUBIN))sym("nvrtcGetCUBIN");
      api.DestroyProgram = (decltype(api.DestroyProgram))sym("nvrtcDestroyProgram");
      if (api.Version && api.CreateProgram && api.CompileProgram && api.GetProgramLogSize && api.GetProgramLog &&
          api.GetCUBINSize && api.GetCUBIN && api.DestroyProgram) {
        api.path = n;
        return;
      }
      api = NvrtcApi();
    }
  });
  if (!api.Version) fail(FGT_ERR_COMPILE, "NVRTC (libnvrtc.so.12) could not be loaded; set FGT_NVRTC to its path");
  return api;
}

Compiled compile_cubin(const std::string& name, const std::string& src, const std::string& cache_dir) {
  int maj = 0, min = 0;
  const NvrtcApi& nv = nvrtc();
  nv.Version(&maj, &min);
  std::string opts;
  for (const char* o : kNvrtcOptions) opts += o, opts += ' ';
  const std::string key = std::to_string(maj) + "." + std::to_string(min) + "|" + opts + "|" + src;
  const std::string digest = sha256_hex(key) + "\n";
  char hex[32];
  std::snprintf(hex, sizeof hex, "%016llx", (unsigned long long)fnv1a(key));
  std::string path;
  Compiled c;
  for (int slot = 0; slot < 8; ++slot) {
    path = cache_dir + "/" + name + "-" + hex + (slot ? "-" + std::to_string(slot) : std::string()) + ".cubin";
    const std::string stored = read_file(path + ".key");
    if (stored.empty()) break;                  // free slot (or an entry without its digest: rebuilt)
    if (stored != digest) continue;             // another key with the same 64-bit hash
    c.cubin = read_file(path);
    if (c.cubin.empty()) break;
    std::string info = read_file(path + ".regs");
    if (!info.empty()) std::sscanf(info.c_str(), "%d %d", &c.regs, &c.spill_bytes);
    return c;
  }
  nvrtcProgram prog;
  if (nv.CreateProgram(&prog, src.c_str(), (name + ".cu").c_str(), 0, nullptr, nullptr) != NVRTC_SUCCESS)
    fail(FGT_ERR_COMPILE, "nvrtcCreateProgram failed for " + name);
  nvrtcResult r = nv.CompileProgram(prog, (int)(sizeof kNvrtcOptions / sizeof kNvrtcOptions[0]), kNvrtcOptions);
  size_t log_size = 0;
  nv.GetProgramLogSize(prog, &log_size);
  std::string log(log_size, '\0');
  if (log_size) nv.GetProgramLog(prog, &log[0]);
  if (r != NVRTC_SUCCESS) {
    nv.DestroyProgram(&prog);
    fail(FGT_ERR_COMPILE, "kernel " + name + " failed to compile: " + log);
  }
  size_t n = 0;
  nv.GetCUBINSize(prog, &n);
  c.cubin.assign(n, '\0');
  nv.GetCUBIN(prog, &c.cubin[0]);
  nv.DestroyProgram(&prog);
  parse_ptxas_report(log, &c);
  mkdirs(cache_dir);
  publish(path + ".regs", std::to_string(c.regs) + " " + std::to_string(c.spill_bytes) + "\n");
  publish(path, c.cubin);
  publish(path + ".key", digest);  // last: the entry counts only once it is complete
  return c;
}

// ---------------------------------------------------------------- NCCL ----
// NCCL is opened at run time so that the process keeps whichever libnccl the
// host framework already loaded (torch bundles its own).
typedef int nccl_result;
typedef void* nccl_comm;
constexpr nccl_result kNcclInProgress = 7;  // ncclInProgress

// The communicator configuration in the layout of NCCL 2.17 (every later
// NCCL reads a configuration by its declared size and version); only
// `blocking` is set, the rest keep NCCL's defaults (the "undefined" values).
struct CommConfig217 {
  size_t size = sizeof(CommConfig217);
  unsigned int magic = 0xcafebeef;
  unsigned int version = 21700;  // NCCL_VERSION(2, 17, 0)
  int blocking = 0;
  int cgaClusterSize = INT_MIN;
  int minCTAs = INT_MIN;
  int maxCTAs = INT_MIN;
  const char* netName = nullptr;
  int splitShare = INT_MIN;
};

struct NcclApi {
  bool ok = false;
  std::string err;
  nccl_result (*GetUniqueId)(void*) = nullptr;
  nccl_result (*CommInitRankConfig)(nccl_comm*, int, const void* /*ncclUniqueId by value*/, int, CommConfig217*) = nullptr;
  nccl_result (*CommDestroy)(nccl_comm) = nullptr;
  nccl_result (*CommAbort)(nccl_comm) = nullptr;
  nccl_result (*CommGetAsyncError)(nccl_comm, nccl_result*) = nullptr;
  nccl_result (*AllGather)(const void*, void*, size_t, int, nccl_comm, void*) = nullptr;
  nccl_result (*AllReduce)(const void*, void*, size_t, int, int, nccl_comm, void*) = nullptr;
  const char* (*GetErrorString)(nccl_result) = nullptr;
};

struct UniqueId {
  char internal[128];
};
typedef nccl_result (*InitRankConfigFn)(nccl_comm*, int, UniqueId, int, CommConfig217*);

NcclApi& nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
      api.err = std::string("cannot load libnccl.so.2: ") + dlerror();
      return;
    }
    api.GetUniqueId = (nccl_result(*)(void*))dlsym(h, "ncclGetUniqueId");
    api.CommInitRankConfig =
        (nccl_result(*)(nccl_comm*, int, const void*, int, CommConfig217*))dlsym(h, "ncclCommInitRankConfig");
    api.CommDestroy = (nccl_result(*)(nccl_comm))dlsym(h, "ncclCommDestroy");
    api.CommAbort = (nccl_result(*)(nccl_comm))dlsym(h, "ncclCommAbort");
    api.CommGetAsyncError = (nccl_result(*)(nccl_comm, nccl_result*))dlsym(h, "ncclCommGetAsyncError");
    api.AllGather = (nccl_result(*)(const void*, void*, size_t, int, nccl_comm, void*))dlsym(h, "ncclAllGather");
    api.AllReduce = (nccl_result(*)(const void*, void*, size_t, int, int, nccl_comm, void*))dlsym(h, "ncclAllReduce");
    api.GetErrorString = (const char* (*)(nccl_result))dlsym(h, "ncclGetErrorString");
    api.ok = api.GetUniqueId && api.CommInitRankConfig && api.CommDestroy && api.CommAbort && api.CommGetAsyncError &&
             api.AllGather && api.AllReduce && api.GetErrorString;
    if (!api.ok) api.err = "libnccl.so.2 lacks a required symbol (NCCL >= 2.17 is needed)";
  });
  return api;
}

void nccl_check(nccl_result r, const char* what) {
  if (r != 0 && r != kNcclInProgress) fail(FGT_ERR_NCCL, std::string(what) + ": " + nccl().GetErrorString(r));
}

// Deadline of a communicator's host-side waits (initialisation, and each
// collective's enqueue on the non-blocking communicator): FGT_COMM_TIMEOUT_MS,
// default 300 s.
int64_t comm_timeout_ms() {
  if (const char* t = std::getenv("FGT_COMM_TIMEOUT_MS")) {
    const long long v = std::atoll(t);
    if (v > 0) return v;
  }
  return 300000;
}

// Wait until a non-blocking communicator leaves ncclInProgress. On an error
// or when the deadline passes the communicator is aborted (it is unusable
// afterwards) and FGT_ERR_NCCL is raised.
void nccl_wait(nccl_comm& comm, const char* what) {
  const auto t0 = std::chrono::steady_clock::now();
  const int64_t limit = comm_timeout_ms();
  for (;;) {
    nccl_result state = 0;
    const nccl_result r = nccl().CommGetAsyncError(comm, &state);
    if (r != 0) state = r;
    if (state == 0) return;
    const int64_t waited =
        std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0).count();
    if (state != kNcclInProgress || waited >= limit) {
      nccl().CommAbort(comm);
      comm = nullptr;
      if (state != kNcclInProgress) fail(FGT_ERR_NCCL, std::string(what) + ": " + nccl().GetErrorString(state));
      fail(FGT_ERR_NCCL, std::string(what) + ": timed out after " + std::to_string(waited) +
                             " ms (FGT_COMM_TIMEOUT_MS); communicator aborted");
    }
    std::this_thread::sleep_for(std::chrono::microseconds(200));
  }
}

}  // namespace

// ------------------------------------------------------------------ spec ---
struct LoadedModule {
  std::vector<CUmodule> mods;
  std::vector<CUfunction> fn;
  std::vector<int> occupancy;  // resident CTAs per SM
  int sms = 0;
};

}  // namespace fgt

struct fgt_spec {
  fgt::Plan plan;
  std::vector<std::string> cubins;
  std::mutex mu;
  std::map<CUcontext, fgt::LoadedModule> modules;
  std::string json;
};

struct fgt_comm {
  fgt::nccl_comm comm = nullptr;
  int world = 1, rank = 0;
  // Peer mailboxes (reductions over the sharded dimension exchange their
  // records with NVLink stores instead of an NCCL all-gather): this rank's
  // mailbox, every rank's mailbox mapped here (own included), and a status
  // word in host-mapped memory that a timed-out exchange sets.
  bool p2p = false;
  CUdeviceptr mailbox = 0;
  CUdeviceptr peers[fgt::kXMaxWorld] = {};
  unsigned* status_host = nullptr;
  CUdeviceptr status_dev = 0;
  unsigned long long wait_limit_ns = 10000000000ull;
};

// A prepared program: per CUDA context, the spec's kernels as one
// instantiated CUDA graph (a chain of kernel nodes in launch order).
struct fgt_program {
  fgt_spec* spec = nullptr;
  bool use_graph = true;
  std::mutex mu;
  struct Instance {
    CUgraph graph = nullptr;
    CUgraphExec exec = nullptr;
    std::vector<CUgraphNode> nodes;
  };
  std::map<CUcontext, Instance> instances;
  ~fgt_program() {
    for (auto& kv : instances) {
      if (kv.second.exec) fgt::drv().GraphExecDestroy(kv.second.exec);
      if (kv.second.graph) fgt::drv().GraphDestroy(kv.second.graph);
    }
  }
};

namespace fgt {
namespace {

int current_sm_count() {
  if (!drv().ok) return 0;
  CUcontext ctx = nullptr;
  if (drv().CtxGetCurrent(&ctx) != CUDA_SUCCESS || !ctx) return 0;
  CUdevice dev;
  if (drv().CtxGetDevice(&dev) != CUDA_SUCCESS) return 0;
  int sms = 0;
  drv().DeviceGetAttribute(&sms, CU_DEVICE_ATTRIBUTE_MULTIPROCESSOR_COUNT, dev);
  return sms;
}

CUcontext ensure_context() {
  require(drv().ok, drv().err, FGT_ERR_CUDA);
  CUcontext ctx = nullptr;
  CUresult r = drv().CtxGetCurrent(&ctx);
  if (r == CUDA_ERROR_NOT_INITIALIZED) {
    cu_check(drv().Init(0), "cuInit");
    r = drv().CtxGetCurrent(&ctx);
  }
  cu_check(r, "cuCtxGetCurrent");
  if (!ctx) {
    CUdevice dev;
    cu_check(drv().DeviceGet(&dev, 0), "cuDeviceGet");
    cu_check(drv().DevicePrimaryCtxRetain(&ctx, dev), "cuDevicePrimaryCtxRetain");
    cu_check(drv().CtxSetCurrent(ctx), "cuCtxSetCurrent");
  }
  return ctx;
}

LoadedModule& module_for(fgt_spec* s) {
  CUcontext ctx = ensure_context();
  std::lock_guard<std::mutex> lock(s->mu);
  auto it = s->modules.find(ctx);
  if (it != s->modules.end()) return it->second;
  LoadedModule lm;
  CUdevice dev;
  cu_check(drv().CtxGetDevice(&dev), "cuCtxGetDevice");
  cu_check(drv().DeviceGetAttribute(&lm.sms, CU_DEVICE_ATTRIBUTE_MULTIPROCESSOR_COUNT, dev), "cuDeviceGetAttribute");
  int major = 0;
  cu_check(drv().DeviceGetAttribute(&major, CU_DEVICE_ATTRIBUTE_COMPUTE_CAPABILITY_MAJOR, dev), "cuDeviceGetAttribute");
  if (major != 10) fail(FGT_ERR_CUDA, "fgt kernels are built for sm_100a (B200); the current device is sm_" + std::to_string(major) + "x");
  // One module per kernel keeps each cubin independent of the others.
  for (size_t i = 0; i < s->plan.kernels.size(); ++i) {
    CUmodule m;
    cu_check(drv().ModuleLoadData(&m, s->cubins[i].data()), "cuModuleLoadData");
    CUfunction f;
    cu_check(drv().ModuleGetFunction(&f, m, s->plan.kernels[i].name.c_str()), "cuModuleGetFunction");
    const int smem = (int)s->plan.kernels[i].smem_bytes;
    // Dynamic plus static shared memory above 48 KB needs the opt-in; set it
    // for every kernel with a ring (static reduction buffers come on top).
    if (smem > 0)
      cu_check(drv().FuncSetAttribute(f, CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES, smem), "cuFuncSetAttribute");
    int occ = 1;
    const KernelDef& kd = s->plan.kernels[i];
    if (drv().OccupancyMaxActiveBlocksPerMultiprocessor(&occ, f, kd.nt, (size_t)smem) != CUDA_SUCCESS || occ < 1) {
      // estimate from the compile report (cluster kernels may not answer the query)
      occ = kd.regs > 0 ? std::max(1, 65536 / (kd.regs * kd.nt)) : 1;
      if (smem > 0) occ = std::max(1, std::min<int>(occ, (int)((227 * 1024) / (smem + 1024))));
    }
    lm.mods.push_back(m);
    lm.fn.push_back(f);
    lm.occupancy.push_back(std::max(1, occ));
  }
  return s->modules.emplace(ctx, std::move(lm)).first->second;
}

struct ArgBlock {
  std::vector<unsigned char> bytes;
};

ArgBlock make_args(const Plan& p, const void* const* inputs, void* const* outputs, void* ws, long long nparts,
                   const fgt_comm* xcomm = nullptr) {
  const int nin = std::max<int>(1, (int)p.g.input_nodes.size());
  const int nout = std::max<int>(1, (int)p.g.outputs.size());
  ArgBlock a;
  const size_t base = (size_t)(nin + nout + 3) * 8;
  a.bytes.assign(base + (xcomm ? (size_t)(kXMaxWorld + 3) * 8 : 0), 0);
  unsigned char* b = a.bytes.data();
  for (size_t i = 0; i < p.g.input_nodes.size(); ++i) std::memcpy(b + 8 * i, &inputs[i], 8);
  for (size_t i = 0; i < p.g.outputs.size(); ++i) std::memcpy(b + 8 * (nin + i), &outputs[i], 8);
  std::memcpy(b + 8 * (nin + nout), &ws, 8);
  std::memcpy(b + 8 * (nin + nout + 1), &nparts, 8);
  if (xcomm) {
    // peer-exchange FIN kernels: xmb[kXMaxWorld], xstat, xrank, xlimit
    unsigned char* x = b + base;
    for (int k = 0; k < kXMaxWorld; ++k) std::memcpy(x + 8 * k, &xcomm->peers[k], 8);
    std::memcpy(x + 8 * kXMaxWorld, &xcomm->status_dev, 8);
    const long long rank = xcomm->rank;
    std::memcpy(x + 8 * (kXMaxWorld + 1), &rank, 8);
    std::memcpy(x + 8 * (kXMaxWorld + 2), &xcomm->wait_limit_ns, 8);
  }
  return a;
}

int64_t grid_for(const KernelDef& k, const LoadedModule& lm, size_t idx) {
  const int64_t resident = (int64_t)lm.sms * lm.occupancy[idx];
  switch (k.kind) {
    case KKind::ROW: {
      // a cluster of k.cluster CTAs per row group; the grid is a whole number of clusters
      int64_t groups = (k.dom.NR + k.rows_per_cta - 1) / k.rows_per_cta;
      // column tiles (gridDim.y) share the resident CTAs
      int64_t g = std::min(groups * k.cluster, std::max<int64_t>(1, resident / std::max<int64_t>(1, k.col_tiles)));
      if (k.max_ctas > 0) g = std::min(g, k.max_ctas * k.cluster);
      g = std::max<int64_t>(k.cluster, g / k.cluster * k.cluster);
      // Balanced waves: CTA i takes row groups i, i + G, ...; when the groups are
      // not a whole number of rounds, the last round runs with only part of the
      // CTAs. Keep the number of rounds and shrink G so that every CTA gets the
      // same number of groups, or one fewer (e.g. 2048 groups on 592 resident
      // CTAs: 512 CTAs x 4 instead of 272 x 4 + 320 x 3).
      const int64_t ctas = g / k.cluster;
      const int64_t rounds = (groups + ctas - 1) / ctas;
      g = std::max<int64_t>(1, (groups + rounds - 1) / rounds) * k.cluster;
      return g;
    }
    case KKind::ELEM: {
      int64_t chunks = k.dom.NI / std::max(1, k.vec);
      int64_t need = (chunks + k.nt - 1) / k.nt;
      int64_t g = std::min(need, resident);
      if (k.max_ctas > 0) g = std::min(g, k.max_ctas);
      return g;
    }
    case KKind::COLFIN:
      // the peer-exchange form pairs CTA c with CTA c of every rank: the same
      // grid on every rank, all CTAs resident, at most kXMaxCtas flags
      // stage 2 walks columns one per thread; the others take blocks of 32 columns
      if (k.fin_stage == 3) return std::max<int64_t>(1, std::min<int64_t>({(k.dom.NI + 31) / 32, (int64_t)lm.sms, (int64_t)kXMaxCtas}));
      if (k.fin_stage == 2) return std::max<int64_t>(1, std::min<int64_t>((k.dom.NI + k.nt - 1) / k.nt, (int64_t)lm.sms * 4));
      return std::max<int64_t>(1, std::min<int64_t>((k.dom.NI + 31) / 32, (int64_t)lm.sms * 4));
    case KKind::FULLFIN:
      return 1;
  }
  return 1;
}

bool empty_kernel(const KernelDef& k) {
  if (k.kind == KKind::ELEM) return k.dom.NI == 0;
  if (k.kind == KKind::ROW) return k.dom.NR == 0;
  if (k.kind == KKind::COLFIN) return k.dom.NI == 0;
  return false;
}

void check_ptr(const void* p, int64_t bytes, const std::string& what) {
  if (bytes == 0) return;
  require(p != nullptr, what + " is NULL");
  require(((uintptr_t)p % 16) == 0, what + " must be 16-byte aligned");
}

// One kernel launch of a spec: the kernel, its grid, and the partial count
// of the kernel whose partials it combines (0 if none).
struct Step {
  size_t idx;
  unsigned grid, gy;
  long long nparts;
};

// path: 1 = NCCL (FIN stages 1 and 2 around the all-gather), 2 = peer
// mailboxes (FIN stage 3); kernels of the other path are not launched.
std::vector<Step> plan_steps(const Plan& p, const LoadedModule& lm, int path = 1) {
  std::vector<Step> steps;
  std::vector<int64_t> parts(p.kernels.size(), 0);
  for (size_t i = 0; i < p.kernels.size(); ++i) {
    const KernelDef& k = p.kernels[i];
    long long nparts = 0;
    if (k.producer >= 0) nparts = parts[k.producer];
    if (empty_kernel(k)) continue;
    if (k.path != 0 && k.path != path) continue;
    int64_t grid = grid_for(k, lm, i);
    parts[i] = k.kind == KKind::ROW ? grid / k.cluster * k.rows_per_cta : grid;
    const unsigned gy = k.kind == KKind::ROW ? (unsigned)std::max<int64_t>(1, k.col_tiles) : 1u;
    steps.push_back(Step{i, (unsigned)grid, gy, nparts});
  }
  return steps;
}

void validate_buffers(const Plan& p, const void* const* inputs, void* const* outputs, void* ws, size_t ws_bytes) {
  require((int64_t)ws_bytes >= p.workspace_bytes, "workspace of " + std::to_string(ws_bytes) + " bytes is smaller than the " +
                                                      std::to_string(p.workspace_bytes) + " bytes the partition needs",
          FGT_ERR_WORKSPACE);
  if (p.workspace_bytes > 0) require(ws != nullptr && ((uintptr_t)ws % 256) == 0, "workspace must be a 256-byte aligned device buffer", FGT_ERR_WORKSPACE);
  for (size_t i = 0; i < p.g.input_nodes.size(); ++i) {
    const Node& n = p.g.nodes[p.g.input_nodes[i]];
    check_ptr(inputs ? inputs[i] : nullptr, n.n() * dtype_size(n.dt), "input " + std::to_string(i));
  }
  for (size_t i = 0; i < p.g.outputs.size(); ++i) {
    const Node& n = p.g.nodes[p.g.outputs[i]];
    check_ptr(outputs ? outputs[i] : nullptr, n.n() * dtype_size(n.dt), "output " + std::to_string(i));
  }
}

// FGT_PDL=0: every kernel launched with plain stream order
bool pdl_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("FGT_PDL");
    return !(e && std::atoi(e) == 0);
  }();
  return on;
}

void launch_all(fgt_spec* s, fgt_comm* comm, const void* const* inputs, void* const* outputs, void* ws, size_t ws_bytes,
                void* stream) {
  const Plan& p = s->plan;
  validate_buffers(p, inputs, outputs, ws, ws_bytes);
  bool xpath = false;
  if (!p.collectives.empty()) {
    require(comm != nullptr, "this spec reduces over the sharded dimension: launch it with fgt_spec_launch_sharded");
    require(comm->world == p.opt.world && comm->rank == p.opt.rank, "communicator rank/world differ from the spec's shard options");
    // a communicator that failed or timed out earlier launches nothing
    require(comm->comm != nullptr, "the communicator failed earlier and was aborted", FGT_ERR_NCCL);
    nccl_result state = 0;
    nccl_check(nccl().CommGetAsyncError(comm->comm, &state), "ncclCommGetAsyncError");
    require(state == 0, std::string("communicator error before launch: ") + nccl().GetErrorString(state), FGT_ERR_NCCL);
    require(!comm->status_host || *(volatile unsigned*)comm->status_host == 0,
            "an earlier peer exchange on this communicator timed out (a rank did not arrive within "
            "FGT_EXCHANGE_WAIT_MS); its results are invalid",
            FGT_ERR_NCCL);
    for (const KernelDef& k : p.kernels) xpath = xpath || (k.path == 2 && comm->p2p);
  }
  LoadedModule& lm = module_for(s);
  CUstream st = (CUstream)stream;
  // Kernels are launched with programmatic stream serialization: each may be
  // scheduled while the kernel before it on the stream drains, and every
  // generated kernel waits for that predecessor to complete, with its memory
  // visible (griddepcontrol.wait), before it reads anything, whichever kernel
  // the predecessor is. Plain launches remain for the kernel after an NCCL
  // collective, for every kernel while the stream is being captured into a
  // graph, and for sharded launches (the cross-rank exchange keeps the stream
  // order its multi-GPU runs were measured with).
  bool pdl = pdl_enabled() && drv().LaunchKernelEx != nullptr && comm == nullptr;
  if (pdl && drv().StreamIsCapturing) {
    CUstreamCaptureStatus cs = CU_STREAM_CAPTURE_STATUS_NONE;
    pdl = drv().StreamIsCapturing(st, &cs) == CUDA_SUCCESS && cs == CU_STREAM_CAPTURE_STATUS_NONE;
  }
  bool after_collective = false;
  for (const Step& sp : plan_steps(p, lm, xpath ? 2 : 1)) {
    const size_t i = sp.idx;
    const KernelDef& k = p.kernels[i];
    ArgBlock a = make_args(p, inputs, outputs, ws, sp.nparts, k.fin_stage == 3 ? comm : nullptr);
    void* params[] = {a.bytes.data()};
    if (pdl && !after_collective) {
      CUlaunchAttribute at[1] = {};
      at[0].id = CU_LAUNCH_ATTRIBUTE_PROGRAMMATIC_STREAM_SERIALIZATION;
      at[0].value.programmaticStreamSerializationAllowed = 1;
      CUlaunchConfig cfg = {};
      cfg.gridDimX = sp.grid;
      cfg.gridDimY = sp.gy;
      cfg.gridDimZ = 1;
      cfg.blockDimX = (unsigned)k.nt;
      cfg.blockDimY = 1;
      cfg.blockDimZ = 1;
      cfg.sharedMemBytes = (unsigned)k.smem_bytes;
      cfg.hStream = st;
      cfg.attrs = at;
      cfg.numAttrs = 1;
      cu_check(drv().LaunchKernelEx(&cfg, lm.fn[i], params, nullptr), "cuLaunchKernelEx");
    } else {
      cu_check(drv().LaunchKernel(lm.fn[i], sp.grid, sp.gy, 1, (unsigned)k.nt, 1, 1, (unsigned)k.smem_bytes, st, params,
                                  nullptr),
               "cuLaunchKernel");
    }
    after_collective = false;
    for (int c : p.collectives) {
      if (c != (int)i || xpath) continue;
      unsigned char* base = (unsigned char*)ws;
      nccl_check(nccl().AllGather(base + k.send_offset, base + k.recv_offset, (size_t)k.record_bytes, /*ncclChar*/ 0,
                                  comm->comm, stream),
                 "ncclAllGather");
      nccl_wait(comm->comm, "ncclAllGather");
      after_collective = true;
    }
  }
}

template <class F>
fgt_status guarded(F&& f) {
  try {
    f();
    return FGT_OK;
  } catch (const Error& e) {
    return set_error(e.status, e.what());
  } catch (const std::exception& e) {
    return set_error(FGT_ERR_INVALID, e.what());
  }
}

fgt_status copy_out(const std::string& s, char* buffer, size_t capacity, size_t* needed) {
  if (needed) *needed = s.size() + 1;
  if (buffer && capacity) {
    size_t n = std::min(capacity - 1, s.size());
    std::memcpy(buffer, s.data(), n);
    buffer[n] = 0;
  }
  return FGT_OK;
}

}  // namespace

// Status + thread-local message for entry points defined in other files.
fgt_status record_error(fgt_status s, const std::string& m) { return set_error(s, m); }

}  // namespace fgt

using namespace fgt;

extern "C" {

const char* fgt_last_error(void) { return g_last_error.c_str(); }

int32_t fgt_abi_version(void) { return FGT_ABI_VERSION; }

fgt_status fgt_spec_create(const fgt_partition_desc* desc, const fgt_spec_options* options, fgt_spec** out) {
  if (!out) return set_error(FGT_ERR_INVALID, "out is NULL");
  *out = nullptr;
  return guarded([&] {
    Graph g = build_graph(desc);
    Options opt;
    const char* cache_dir = nullptr;
    if (options) {
      require(options->accumulation == FGT_ACCUM_WIDE || options->accumulation == FGT_ACCUM_STORAGE, "unknown accumulation policy");
      opt.accumulation = options->accumulation;
      if (options->shard_world > 1) {
        require(options->shard_rank >= 0 && options->shard_rank < options->shard_world, "shard_rank out of range");
        opt.world = options->shard_world;
        opt.rank = options->shard_rank;
        opt.shard_inputs = options->shard_inputs;
      }
      cache_dir = options->cache_dir;
      require(options->row_elems >= 0 && options->row_elems <= 64, "row_elems must be in [0, 64]");
      require(options->ring_kb >= 0 && options->ring_kb <= 200, "ring_kb must be in [0, 200]");
      if (options->row_elems > 0) opt.row_elems = options->row_elems;
      if (options->ring_kb > 0) opt.ring_kb = options->ring_kb;
      require(options->row_cluster >= 0 && options->row_cluster <= 8 && (options->row_cluster & (options->row_cluster - 1)) == 0,
              "row_cluster must be 0 or a power of two up to 8");
      if (options->row_cluster > 0) opt.row_cluster = options->row_cluster;
      require((options->row_flags & ~(FGT_ROW_OCCUPANCY_STEP | FGT_ROW_EXPF | FGT_ROW_SMEM_COLS | FGT_ROW_XW_SHUFFLE |
                                      FGT_ROW_RING_RESIDENT | FGT_ROW_PHASE_COPIES | FGT_ROW_PACK_COLS |
                                      FGT_ROW_TMEM_COLS | FGT_ROW_NARROW_DIV)) == 0,
              "unknown row_flags bits");
      opt.phase_copies = (options->row_flags & FGT_ROW_PHASE_COPIES) != 0;
      opt.pack_cols = (options->row_flags & FGT_ROW_PACK_COLS) != 0;
      opt.tmem_cols = (options->row_flags & FGT_ROW_TMEM_COLS) != 0;
      opt.narrow_div = (options->row_flags & FGT_ROW_NARROW_DIV) != 0;
      opt.ring_resident = (options->row_flags & FGT_ROW_RING_RESIDENT) != 0;
      if (options->row_flags & FGT_ROW_XW_SHUFFLE) opt.xw_tree = 0;
      opt.occupancy_step = (options->row_flags & FGT_ROW_OCCUPANCY_STEP) != 0;
      opt.smem_cols = (options->row_flags & FGT_ROW_SMEM_COLS) != 0;
      if (options->row_flags & FGT_ROW_EXPF) opt.own_exp = 0;
    }
    // FGT_ROW_STAGING=0 keeps streamed row operands in registers
    // (double-buffered) instead of the shared-memory ring.
    if (const char* st = std::getenv("FGT_ROW_STAGING")) opt.row_staging = std::atoi(st) != 0;
    {
      // three-input max / min assemble from NVRTC 12.9 on (PTX ISA 8.8)
      int maj = 0, mnr = 0;
      nvrtc().Version(&maj, &mnr);
      opt.max3 = (maj > 12 || (maj == 12 && mnr >= 9)) ? 1 : 0;
      if (const char* m3 = std::getenv("FGT_MAX3")) opt.max3 = opt.max3 && std::atoi(m3) != 0;
    }
    if (const char* lp = std::getenv("FGT_LANE_PAIRS")) opt.lane_pairs = std::atoi(lp) != 0;
    if (const char* ox = std::getenv("FGT_OWN_EXP")) opt.own_exp = std::atoi(ox) != 0;
    if (const char* xs = std::getenv("FGT_XW_SHUFFLE")) opt.xw_tree = std::atoi(xs) == 0;
    bool row_elems_forced = options && options->row_elems > 0;
    if (const char* re = std::getenv("FGT_ROW_ELEMS")) {
      opt.row_elems = std::max(1, std::min(64, std::atoi(re)));
      row_elems_forced = true;
    }
    if (const char* rk = std::getenv("FGT_RING_KB")) opt.ring_kb = std::max(4, std::min(200, std::atoi(rk)));
    if (const char* rc = std::getenv("FGT_ROW_CLUSTER")) {
      const int v = std::atoi(rc);
      if (v == 1 || v == 2 || v == 4) opt.row_cluster = v;
    }
    int sms = current_sm_count();
    if (sms > 0) opt.num_sms = sms;
    auto spec = std::make_unique<fgt_spec>();
    const std::string dir = cache_root(cache_dir);
    auto specialise = [&](const Options& o, Plan* plan, std::vector<std::string>* cubins) {
      *plan = make_plan(g, o);
      generate_sources(*plan);
      cubins->clear();
      for (auto& k : plan->kernels) {
        // FGT_DUMP_DIR: write each kernel's generated source before compiling it (debugging)
        if (const char* dump = std::getenv("FGT_DUMP_DIR")) {
          mkdirs(dump);
          std::ofstream f(std::string(dump) + "/" + k.name + ".cu");
          f << k.source;
        }
        Compiled c = compile_cubin(k.name, std::string(fgt_device_library_source) + "\n" + k.source, dir);
        // Occupancy step: registers are allocated per thread in steps of 8,
        // so a block-per-row kernel a little above a CTA-count boundary (say
        // 79 registers at 256 threads: 3 CTAs per SM) is compiled again bounded
        // to one more CTA per SM (64 registers: 4) when that bound is within
        // 70% of its registers and the ring still fits; kept with at most 256
        // bytes of spills (the option is a tuning candidate: the tuner times
        // it against the unbounded kernel).
        if (o.occupancy_step && k.kind == KKind::ROW && c.regs > 0 && c.spill_bytes == 0) {
          const int64_t per = ((c.regs + 7) / 8) * 8 * (int64_t)k.nt;
          const int64_t ctas = 65536 / per, max_ctas = 2048 / k.nt;
          const int64_t target = ctas + 1, cap = (65536 / (target * k.nt)) / 8 * 8;
          const std::string lb = "__launch_bounds__(" + std::to_string(k.nt) + ")";
          const size_t at = k.source.find(lb);
          if (ctas >= 1 && target <= max_ctas && cap >= 32 && cap * 10 >= (int64_t)c.regs * 7 &&
              k.smem_bytes * target <= 227 * 1024 && at != std::string::npos) {
            std::string src = k.source;
            src.replace(at, lb.size(), "__launch_bounds__(" + std::to_string(k.nt) + ", " + std::to_string(target) + ")");
            Compiled b = compile_cubin(k.name, std::string(fgt_device_library_source) + "\n" + src, dir);
            if (b.spill_bytes >= 0 && b.spill_bytes <= 256 && b.regs > 0 && b.regs <= cap) {
              k.source = src;
              c = std::move(b);
            }
          }
        }
        k.regs = c.regs;
        k.spill_bytes = c.spill_bytes;
        cubins->push_back(std::move(c.cubin));
      }
    };
    specialise(opt, &spec->plan, &spec->cubins);
    // Row geometry from the compile report. A block-per-row kernel of 512
    // threads above 64 registers fits one CTA (16 warps) per SM. With a single
    // barrier phase per row and no column partials, 8 elements per thread
    // (1024 threads) then runs faster (measured on the broadcast-select
    // workload: 74 -> 40 registers, 0.51 -> 0.62 of HBM peak); kernels with
    // more phases lose more to the extra barriers per element than they gain.
    if (!row_elems_forced && opt.row_elems > 8) {
      bool retry = false;
      for (auto& k : spec->plan.kernels) {
        bool col = false;
        for (auto& rd : k.reds) col = col || rd.role == ROLE_COL;
        if (k.kind == KKind::ROW && k.tpr >= 512 && k.nt == 512 && k.regs > 64 && k.row_phases <= 1 && !col) retry = true;
      }
      if (retry) {
        Options o8 = opt;
        o8.row_elems = 8;
        Plan p8;
        std::vector<std::string> c8;
        specialise(o8, &p8, &c8);
        bool better = true;
        for (auto& k : p8.kernels)
          if (k.kind == KKind::ROW && (k.regs < 0 || k.regs > 64 || k.spill_bytes != 0)) better = false;
        if (better) {
          spec->plan = std::move(p8);
          spec->cubins = std::move(c8);
        }
      }
    }
    spec->json = plan_json(spec->plan);
    *out = spec.release();
  });
}

void fgt_spec_destroy(fgt_spec* spec) {
  if (!spec) return;
  for (auto& [ctx, lm] : spec->modules) {
    if (!drv().ok) break;
    // Modules are released only if their context is still alive.
    CUcontext cur = nullptr;
    if (drv().CtxGetCurrent(&cur) == CUDA_SUCCESS && cur == ctx)
      for (CUmodule m : lm.mods) drv().ModuleUnload(m);
  }
  delete spec;
}

fgt_status fgt_spec_get_info(const fgt_spec* spec, fgt_spec_info* info) {
  if (!spec || !info) return set_error(FGT_ERR_INVALID, "spec or info is NULL");
  info->num_inputs = (int32_t)spec->plan.g.input_nodes.size();
  info->num_outputs = (int32_t)spec->plan.g.outputs.size();
  info->kernel_count = (int32_t)spec->plan.kernels.size();
  info->collective_count = (int32_t)spec->plan.collectives.size();
  info->workspace_bytes = (size_t)spec->plan.workspace_bytes;
  return FGT_OK;
}

fgt_status fgt_spec_port(const fgt_spec* spec, int32_t is_output, int32_t index, int32_t* dtype, int32_t* rank,
                         int64_t* shape) {
  if (!spec) return set_error(FGT_ERR_INVALID, "spec is NULL");
  const Graph& g = spec->plan.g;
  int node;
  if (is_output) {
    if (index < 0 || index >= (int)g.outputs.size()) return set_error(FGT_ERR_INVALID, "output port out of range");
    node = g.outputs[index];
  } else {
    if (index < 0 || index >= (int)g.input_nodes.size()) return set_error(FGT_ERR_INVALID, "input port out of range");
    node = g.input_nodes[index];
  }
  const Node& n = g.nodes[node];
  if (dtype) *dtype = n.dt;
  if (rank) *rank = n.rank();
  if (shape)
    for (int k = 0; k < n.rank(); ++k) shape[k] = n.shape[k];
  return FGT_OK;
}

fgt_status fgt_spec_plan_json(const fgt_spec* spec, char* buffer, size_t capacity, size_t* needed) {
  if (!spec) return set_error(FGT_ERR_INVALID, "spec is NULL");
  return copy_out(spec->json, buffer, capacity, needed);
}

fgt_status fgt_spec_kernel_source(const fgt_spec* spec, int32_t index, char* buffer, size_t capacity, size_t* needed) {
  if (!spec) return set_error(FGT_ERR_INVALID, "spec is NULL");
  if (index < 0 || index >= (int)spec->plan.kernels.size()) return set_error(FGT_ERR_INVALID, "kernel index out of range");
  return copy_out(spec->plan.kernels[index].source, buffer, capacity, needed);
}

fgt_status fgt_spec_launch(const fgt_spec* spec, const void* const* inputs, void* const* outputs, void* workspace,
                           size_t workspace_bytes, void* stream) {
  if (!spec) return set_error(FGT_ERR_INVALID, "spec is NULL");
  return guarded([&] { launch_all(const_cast<fgt_spec*>(spec), nullptr, inputs, outputs, workspace, workspace_bytes, stream); });
}

fgt_status fgt_program_create(const fgt_spec* spec, int32_t use_graph, fgt_program** out) {
  if (!out) return set_error(FGT_ERR_INVALID, "out is NULL");
  *out = nullptr;
  if (!spec) return set_error(FGT_ERR_INVALID, "spec is NULL");
  return guarded([&] {
    require(spec->plan.collectives.empty(),
            "this spec reduces over the sharded dimension: launch it with fgt_spec_launch_sharded", FGT_ERR_UNSUPPORTED);
    auto p = std::make_unique<fgt_program>();
    p->spec = const_cast<fgt_spec*>(spec);
    p->use_graph = use_graph != 0;
    *out = p.release();
  });
}

fgt_status fgt_program_run(fgt_program* program, const void* const* inputs, void* const* outputs, void* workspace,
                           size_t workspace_bytes, void* stream) {
  if (!program) return set_error(FGT_ERR_INVALID, "program is NULL");
  return guarded([&] {
    fgt_spec* s = program->spec;
    const Plan& p = s->plan;
    // Inside a stream capture a graph launch is not allowed: the kernels are
    // launched one by one and become nodes of the caller's captured graph.
    CUstreamCaptureStatus cap = CU_STREAM_CAPTURE_STATUS_NONE;
    if (program->use_graph && drv().graphs) {
      ensure_context();
      cu_check(drv().StreamIsCapturing((CUstream)stream, &cap), "cuStreamIsCapturing");
    }
    if (!program->use_graph || !drv().graphs || cap != CU_STREAM_CAPTURE_STATUS_NONE) {
      launch_all(s, nullptr, inputs, outputs, workspace, workspace_bytes, stream);
      return;
    }
    validate_buffers(p, inputs, outputs, workspace, workspace_bytes);
    LoadedModule& lm = module_for(s);
    CUcontext ctx = nullptr;
    cu_check(drv().CtxGetCurrent(&ctx), "cuCtxGetCurrent");
    const std::vector<Step> steps = plan_steps(p, lm);
    std::lock_guard<std::mutex> lock(program->mu);
    fgt_program::Instance& in = program->instances[ctx];
    // kernel-node parameters of this run: the run's buffers in each kernel's
    // argument block (copied by the driver when set)
    std::vector<ArgBlock> args;
    std::vector<void*> kp(steps.size());
    std::vector<CUDA_KERNEL_NODE_PARAMS_v2> np(steps.size());
    args.reserve(steps.size());
    for (size_t j = 0; j < steps.size(); ++j) {
      const Step& sp = steps[j];
      const KernelDef& k = p.kernels[sp.idx];
      args.push_back(make_args(p, inputs, outputs, workspace, sp.nparts));
      kp[j] = args.back().bytes.data();
      CUDA_KERNEL_NODE_PARAMS_v2 q;
      std::memset(&q, 0, sizeof q);
      q.func = lm.fn[sp.idx];
      q.gridDimX = sp.grid;
      q.gridDimY = sp.gy;
      q.gridDimZ = 1;
      q.blockDimX = (unsigned)k.nt;
      q.blockDimY = q.blockDimZ = 1;
      q.sharedMemBytes = (unsigned)k.smem_bytes;
      q.kernelParams = &kp[j];
      np[j] = q;
    }
    if (steps.empty()) return;
    if (!in.exec) {
      cu_check(drv().GraphCreate(&in.graph, 0), "cuGraphCreate");
      CUgraphNode prev = nullptr;
      for (size_t j = 0; j < steps.size(); ++j) {
        CUgraphNode node = nullptr;
        cu_check(drv().GraphAddKernelNode(&node, in.graph, prev ? &prev : nullptr, prev ? 1 : 0, &np[j]),
                 "cuGraphAddKernelNode");
        in.nodes.push_back(node);
        prev = node;
      }
      cu_check(drv().GraphInstantiate(&in.exec, in.graph, 0), "cuGraphInstantiate");
    } else {
      require(in.nodes.size() == steps.size(), "internal: program graph changed shape", FGT_ERR_CUDA);
      for (size_t j = 0; j < steps.size(); ++j)
        cu_check(drv().GraphExecKernelNodeSetParams(in.exec, in.nodes[j], &np[j]), "cuGraphExecKernelNodeSetParams");
    }
    cu_check(drv().GraphLaunch(in.exec, (CUstream)stream), "cuGraphLaunch");
  });
}

int32_t fgt_program_kernel_count(const fgt_program* program) {
  if (!program) return 0;
  int32_t n = 0;
  for (const KernelDef& k : program->spec->plan.kernels) n += empty_kernel(k) ? 0 : 1;
  return n;
}

void fgt_program_destroy(fgt_program* program) { delete program; }

fgt_status fgt_comm_unique_id(uint8_t id[128]) {
  return guarded([&] {
    require(id != nullptr, "id is NULL");
    require(nccl().ok, nccl().err, FGT_ERR_NCCL);
    nccl_check(nccl().GetUniqueId(id), "ncclGetUniqueId");
  });
}

namespace fgt {
namespace {

// All-gather `n` bytes per rank over the communicator (host buffers; for
// set-up and teardown only: it synchronises the context).
void allgather_host(fgt_comm* c, const void* mine, size_t n, void* all) {
  CUdeviceptr buf = 0;
  cu_check(drv().MemAlloc(&buf, n * (size_t)c->world), "cuMemAlloc");
  struct Free {
    CUdeviceptr b;
    ~Free() { drv().MemFree(b); }
  } guard{buf};
  cu_check(drv().MemcpyHtoD(buf + n * (size_t)c->rank, mine, n), "cuMemcpyHtoD");
  nccl_check(nccl().AllGather((const void*)(buf + n * (size_t)c->rank), (void*)buf, n, /*ncclChar*/ 0, c->comm, nullptr),
             "ncclAllGather");
  nccl_wait(c->comm, "ncclAllGather");
  cu_check(drv().CtxSynchronize(), "cuCtxSynchronize");
  cu_check(drv().MemcpyDtoH(all, buf, n * (size_t)c->world), "cuMemcpyDtoH");
}

void release_mailboxes(fgt_comm* c) {
  for (int k = 0; k < kXMaxWorld; ++k)
    if (c->peers[k] && k != c->rank) drv().IpcCloseMemHandle(c->peers[k]);
  for (int k = 0; k < kXMaxWorld; ++k) c->peers[k] = 0;
  if (c->mailbox) drv().MemFree(c->mailbox);
  if (c->status_host) drv().MemFreeHost(c->status_host);
  c->mailbox = 0;
  c->status_host = nullptr;
  c->status_dev = 0;
  c->p2p = false;
}

// Peer mailboxes: every rank allocates one (zeroed) and a host-mapped status
// word, exports the mailbox through CUDA IPC, the handles are all-gathered
// over the communicator, and every rank maps the others'. Used only when
// every rank succeeded at every step (decided together, so all ranks launch
// the same path). FGT_PEER_EXCHANGE=0 keeps the NCCL all-gather path.
void setup_mailboxes(fgt_comm* c) {
  if (const char* e = std::getenv("FGT_PEER_EXCHANGE"))
    if (std::atoi(e) == 0) return;
  if (c->world > kXMaxWorld || !drv().ipc) return;  // the same on every rank of one machine
  if (const char* w = std::getenv("FGT_EXCHANGE_WAIT_MS")) {
    const long long v = std::atoll(w);
    if (v > 0) c->wait_limit_ns = (unsigned long long)v * 1000000ull;
  }
  struct Rec {
    CUipcMemHandle handle;
    int32_t ok;
    char pad[60];
  };
  static_assert(sizeof(Rec) == 128, "mailbox record");
  Rec mine;
  std::memset(&mine, 0, sizeof mine);
  bool ok = drv().MemAlloc(&c->mailbox, (size_t)kXBytes) == CUDA_SUCCESS;
  ok = ok && drv().MemsetD8(c->mailbox, 0, (size_t)kXBytes) == CUDA_SUCCESS;
  ok = ok && drv().IpcGetMemHandle(&mine.handle, c->mailbox) == CUDA_SUCCESS;
  ok = ok && drv().MemHostAlloc((void**)&c->status_host, 64, CU_MEMHOSTALLOC_DEVICEMAP | CU_MEMHOSTALLOC_PORTABLE) ==
                 CUDA_SUCCESS;
  ok = ok && drv().MemHostGetDevicePointer(&c->status_dev, c->status_host, 0) == CUDA_SUCCESS;
  if (ok) *(volatile unsigned*)c->status_host = 0;
  mine.ok = ok ? 1 : 0;
  std::vector<Rec> all((size_t)c->world);
  allgather_host(c, &mine, sizeof(Rec), all.data());
  bool every = true;
  for (const Rec& r : all) every = every && r.ok;
  int32_t opened = every ? 1 : 0;
  for (int k = 0; k < c->world && opened; ++k) {
    if (k == c->rank) continue;
    if (drv().IpcOpenMemHandle(&c->peers[k], all[(size_t)k].handle, CU_IPC_MEM_LAZY_ENABLE_PEER_ACCESS) != CUDA_SUCCESS) {
      c->peers[k] = 0;
      opened = 0;
    }
  }
  std::vector<int32_t> agreed((size_t)c->world);
  allgather_host(c, &opened, sizeof(int32_t), agreed.data());
  for (int32_t a : agreed) every = every && a;
  if (!every) {
    release_mailboxes(c);
    return;
  }
  c->peers[c->rank] = c->mailbox;
  c->p2p = true;
}

}  // namespace
}  // namespace fgt

int32_t fgt_comm_peer_exchange(const fgt_comm* comm) { return comm && comm->p2p ? 1 : 0; }

fgt_status fgt_comm_create(const uint8_t id[128], int32_t world, int32_t rank, fgt_comm** out) {
  if (!out) return set_error(FGT_ERR_INVALID, "out is NULL");
  *out = nullptr;
  return guarded([&] {
    require(id != nullptr && world >= 1 && rank >= 0 && rank < world, "invalid communicator arguments");
    require(nccl().ok, nccl().err, FGT_ERR_NCCL);
    ensure_context();
    auto c = std::make_unique<fgt_comm>();
    c->world = world;
    c->rank = rank;
    UniqueId uid;
    std::memcpy(uid.internal, id, 128);
    // non-blocking: initialisation proceeds in the background and is polled
    // against the deadline, so a rank that never joins ends in an error here
    // instead of a wait without end
    CommConfig217 cfg;
    InitRankConfigFn init = (InitRankConfigFn)(void*)nccl().CommInitRankConfig;
    const nccl_result r = init(&c->comm, world, uid, rank, &cfg);
    if (r != 0 && r != kNcclInProgress) {
      if (c->comm) nccl().CommAbort(c->comm);
      c->comm = nullptr;
      fail(FGT_ERR_NCCL, std::string("ncclCommInitRankConfig: ") + nccl().GetErrorString(r));
    }
    nccl_wait(c->comm, "ncclCommInitRankConfig");
    if (world > 1) {
      try {
        setup_mailboxes(c.get());
      } catch (...) {
        release_mailboxes(c.get());
        if (c->comm) nccl().CommAbort(c->comm);
        c->comm = nullptr;
        throw;
      }
    }
    *out = c.release();
  });
}

void fgt_comm_destroy(fgt_comm* comm) {
  if (!comm) return;
  if (comm->p2p) {
    // No rank unmaps or frees its mailbox while a peer may still write to it:
    // each rank finishes its own work, then all ranks meet. If they cannot
    // meet (a rank is gone or the deadline passed), the mailbox is left
    // mapped rather than freed under a possible writer.
    bool met = false;
    try {
      fgt::cu_check(fgt::drv().CtxSynchronize(), "cuCtxSynchronize");
      int32_t one = 1;
      std::vector<int32_t> all((size_t)comm->world);
      fgt::allgather_host(comm, &one, sizeof one, all.data());
      met = true;
    } catch (...) {
    }
    if (met) fgt::release_mailboxes(comm);
  }
  if (comm->comm && fgt::nccl().ok) fgt::nccl().CommDestroy(comm->comm);
  delete comm;
}

fgt_status fgt_spec_launch_sharded(const fgt_spec* spec, fgt_comm* comm, const void* const* inputs, void* const* outputs,
                                   void* workspace, size_t workspace_bytes, void* stream) {
  if (!spec) return set_error(FGT_ERR_INVALID, "spec is NULL");
  return guarded([&] {
    require(comm != nullptr, "communicator is NULL");
    require(spec->plan.opt.world == comm->world, "spec was not created for this communicator's world size");
    launch_all(const_cast<fgt_spec*>(spec), comm, inputs, outputs, workspace, workspace_bytes, stream);
  });
}

}  // extern "C"
