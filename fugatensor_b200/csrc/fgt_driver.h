// fgt_driver.h — the CUDA driver entry points the runtime uses, opened with
// dlopen on first use. The library therefore loads (and plans / compiles
// partitions with NVRTC) on machines without a GPU driver; only launching
// needs libcuda. Same approach as the reference's driver shim
// (cpp/cuda_driver_api.h:35-98).
#pragma once

#include <cuda.h>
#include <dlfcn.h>

#include <mutex>
#include <string>

namespace fgt {

struct Driver {
  bool ok = false;
  std::string err;
  CUresult (*Init)(unsigned int) = nullptr;
  CUresult (*GetErrorName)(CUresult, const char**) = nullptr;
  CUresult (*GetErrorString)(CUresult, const char**) = nullptr;
  CUresult (*CtxGetCurrent)(CUcontext*) = nullptr;
  CUresult (*CtxSetCurrent)(CUcontext) = nullptr;
  CUresult (*CtxGetDevice)(CUdevice*) = nullptr;
  CUresult (*DeviceGet)(CUdevice*, int) = nullptr;
  CUresult (*DeviceGetAttribute)(int*, CUdevice_attribute, CUdevice) = nullptr;
  CUresult (*DevicePrimaryCtxRetain)(CUcontext*, CUdevice) = nullptr;
  CUresult (*ModuleLoadData)(CUmodule*, const void*) = nullptr;
  CUresult (*ModuleUnload)(CUmodule) = nullptr;
  CUresult (*ModuleGetFunction)(CUfunction*, CUmodule, const char*) = nullptr;
  CUresult (*OccupancyMaxActiveBlocksPerMultiprocessor)(int*, CUfunction, int, size_t) = nullptr;
  CUresult (*FuncSetAttribute)(CUfunction, CUfunction_attribute, int) = nullptr;
  CUresult (*LaunchKernel)(CUfunction, unsigned, unsigned, unsigned, unsigned, unsigned, unsigned, unsigned, CUstream,
                           void**, void**) = nullptr;
  // optional (CUDA 12.0+ drivers): a context's process-unique id
  CUresult (*CtxGetId)(CUcontext, unsigned long long*) = nullptr;
  // optional (CUDA 12.0+ drivers): launches with attributes (programmatic
  // dependent launch of a plan's kernels)
  CUresult (*LaunchKernelEx)(const CUlaunchConfig*, CUfunction, void**, void**) = nullptr;
  // optional: CUDA graphs of prepared programs (kernel-node parameters v2)
  bool graphs = false;
  CUresult (*GraphCreate)(CUgraph*, unsigned int) = nullptr;
  CUresult (*GraphAddKernelNode)(CUgraphNode*, CUgraph, const CUgraphNode*, size_t, const CUDA_KERNEL_NODE_PARAMS_v2*) = nullptr;
  CUresult (*GraphInstantiate)(CUgraphExec*, CUgraph, unsigned long long) = nullptr;
  CUresult (*GraphExecKernelNodeSetParams)(CUgraphExec, CUgraphNode, const CUDA_KERNEL_NODE_PARAMS_v2*) = nullptr;
  CUresult (*GraphLaunch)(CUgraphExec, CUstream) = nullptr;
  CUresult (*GraphExecDestroy)(CUgraphExec) = nullptr;
  CUresult (*GraphDestroy)(CUgraph) = nullptr;
  CUresult (*StreamIsCapturing)(CUstream, CUstreamCaptureStatus*) = nullptr;
  // optional: peer mailboxes of communicators (device memory shared between
  // the ranks' processes through CUDA IPC, and a host-mapped status word)
  bool ipc = false;
  CUresult (*MemAlloc)(CUdeviceptr*, size_t) = nullptr;
  CUresult (*MemFree)(CUdeviceptr) = nullptr;
  CUresult (*MemsetD8)(CUdeviceptr, unsigned char, size_t) = nullptr;
  CUresult (*MemcpyHtoD)(CUdeviceptr, const void*, size_t) = nullptr;
  CUresult (*MemcpyDtoH)(void*, CUdeviceptr, size_t) = nullptr;
  CUresult (*IpcGetMemHandle)(CUipcMemHandle*, CUdeviceptr) = nullptr;
  CUresult (*IpcOpenMemHandle)(CUdeviceptr*, CUipcMemHandle, unsigned int) = nullptr;
  CUresult (*IpcCloseMemHandle)(CUdeviceptr) = nullptr;
  CUresult (*MemHostAlloc)(void**, size_t, unsigned int) = nullptr;
  CUresult (*MemHostGetDevicePointer)(CUdeviceptr*, void*, unsigned int) = nullptr;
  CUresult (*MemFreeHost)(void*) = nullptr;
  CUresult (*CtxSynchronize)() = nullptr;
};

inline Driver& drv() {
  static Driver d;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libcuda.so.1", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
      d.err = std::string("CUDA driver not available (libcuda.so.1): ") + dlerror();
      return;
    }
    bool all = true;
    auto sym = [&](auto& fn, const char* name) {
      fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(h, name));
      all = all && fn != nullptr;
    };
    sym(d.Init, "cuInit");
    sym(d.GetErrorName, "cuGetErrorName");
    sym(d.GetErrorString, "cuGetErrorString");
    sym(d.CtxGetCurrent, "cuCtxGetCurrent");
    sym(d.CtxSetCurrent, "cuCtxSetCurrent");
    sym(d.CtxGetDevice, "cuCtxGetDevice");
    sym(d.DeviceGet, "cuDeviceGet");
    sym(d.DeviceGetAttribute, "cuDeviceGetAttribute");
    sym(d.DevicePrimaryCtxRetain, "cuDevicePrimaryCtxRetain");
    sym(d.ModuleLoadData, "cuModuleLoadData");
    sym(d.ModuleUnload, "cuModuleUnload");
    sym(d.ModuleGetFunction, "cuModuleGetFunction");
    sym(d.OccupancyMaxActiveBlocksPerMultiprocessor, "cuOccupancyMaxActiveBlocksPerMultiprocessor");
    sym(d.LaunchKernel, "cuLaunchKernel");
    sym(d.FuncSetAttribute, "cuFuncSetAttribute");
    d.ok = all;
    if (!all) d.err = "libcuda.so.1 lacks a required driver entry point";
    d.CtxGetId = reinterpret_cast<decltype(d.CtxGetId)>(dlsym(h, "cuCtxGetId"));
    d.LaunchKernelEx = reinterpret_cast<decltype(d.LaunchKernelEx)>(dlsym(h, "cuLaunchKernelEx"));
    auto opt = [&](auto& fn, const char* name) {
      fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(h, name));
      return fn != nullptr;
    };
    bool g = opt(d.GraphCreate, "cuGraphCreate");
    g = opt(d.GraphAddKernelNode, "cuGraphAddKernelNode_v2") && g;
    g = opt(d.GraphInstantiate, "cuGraphInstantiateWithFlags") && g;
    g = opt(d.GraphExecKernelNodeSetParams, "cuGraphExecKernelNodeSetParams_v2") && g;
    g = opt(d.GraphLaunch, "cuGraphLaunch") && g;
    g = opt(d.GraphExecDestroy, "cuGraphExecDestroy") && g;
    g = opt(d.GraphDestroy, "cuGraphDestroy") && g;
    g = opt(d.StreamIsCapturing, "cuStreamIsCapturing") && g;
    d.graphs = g;
    bool ip = opt(d.MemAlloc, "cuMemAlloc_v2");
    ip = opt(d.MemFree, "cuMemFree_v2") && ip;
    ip = opt(d.MemsetD8, "cuMemsetD8_v2") && ip;
    ip = opt(d.MemcpyHtoD, "cuMemcpyHtoD_v2") && ip;
    ip = opt(d.MemcpyDtoH, "cuMemcpyDtoH_v2") && ip;
    ip = opt(d.IpcGetMemHandle, "cuIpcGetMemHandle") && ip;
    ip = opt(d.IpcOpenMemHandle, "cuIpcOpenMemHandle_v2") && ip;
    ip = opt(d.IpcCloseMemHandle, "cuIpcCloseMemHandle") && ip;
    ip = opt(d.MemHostAlloc, "cuMemHostAlloc") && ip;
    ip = opt(d.MemHostGetDevicePointer, "cuMemHostGetDevicePointer_v2") && ip;
    ip = opt(d.MemFreeHost, "cuMemFreeHost") && ip;
    ip = opt(d.CtxSynchronize, "cuCtxSynchronize") && ip;
    d.ipc = ip;
  });
  return d;
}

}  // namespace fgt
