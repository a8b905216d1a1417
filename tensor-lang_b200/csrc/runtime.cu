// Runtime shim: device init, stream-ordered memory pool, copies, streams,
// events, CUDA graphs, NVRTC region JIT and the NCCL loader.
//
// Replaces what the reference takes from PyCUDA (pycuda.autoinit,
// driver.mem_alloc / memcpy_htod / memcpy_dtoh, tensorlang/compiler.py:1472-1503)
// and its per-program `nvcc` + ctypes.cdll step (compiler.py:1429-1476).
#include <cuda.h>
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>
#include <nvrtc.h>

#include <atomic>
#include <chrono>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <mutex>
#include <sstream>
#include <string>
#include <thread>
#include <unordered_map>
#include <vector>

#include "tl_common.cuh"

namespace {

constexpr int kMaxDevices = 64;

struct DeviceState {
  bool ready = false;
  cudaStream_t stream = nullptr;
  int sms = 0;
};

DeviceState g_dev[kMaxDevices];
std::mutex g_mu;
thread_local uint64_t t_launches = 0;
thread_local std::string t_jit_log;

int current_device() {
  int d = 0;
  cudaGetDevice(&d);
  return d;
}

}  // namespace

namespace tl {

cudaStream_t stream_or_default(void* s) {
  if (s) return (cudaStream_t)s;
  int d = current_device();
  return (d >= 0 && d < kMaxDevices) ? g_dev[d].stream : nullptr;
}

int sm_count() {
  int d = current_device();
  if (d >= 0 && d < kMaxDevices && g_dev[d].sms) return g_dev[d].sms;
  int n = 0;
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, d);
  return n > 0 ? n : 148;
}

int after_launch() {
  ++t_launches;
  return (int)cudaGetLastError();
}

}  // namespace tl

extern "C" {

// ---------------------------------------------------------------- device ---
int tl_init(int device) {
  if (device < 0 || device >= kMaxDevices) return TL_ERR_INVALID_ARG;
  TL_CUDA_TRY(cudaSetDevice(device));
  std::lock_guard<std::mutex> lk(g_mu);
  DeviceState& st = g_dev[device];
  if (st.ready) return TL_OK;
  TL_CUDA_TRY(cudaStreamCreateWithFlags(&st.stream, cudaStreamNonBlocking));
  cudaMemPool_t pool;
  TL_CUDA_TRY(cudaDeviceGetDefaultMemPool(&pool, device));
  uint64_t keep = UINT64_MAX;  // cache freed blocks instead of returning them
  TL_CUDA_TRY(cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep));
  TL_CUDA_TRY(cudaDeviceGetAttribute(&st.sms, cudaDevAttrMultiProcessorCount, device));
  st.ready = true;
  return TL_OK;
}

int tl_device_count(int* count) {
  if (!count) return TL_ERR_INVALID_ARG;
  *count = 0;
  cudaError_t e = cudaGetDeviceCount(count);
  if (e != cudaSuccess) {
    *count = 0;
    cudaGetLastError();
    return (int)e;
  }
  return TL_OK;
}

int tl_device_info(int device, int* sm_count, int* cc_major, int* cc_minor, size_t* total_mem) {
  cudaDeviceProp p;
  TL_CUDA_TRY(cudaGetDeviceProperties(&p, device));
  if (sm_count) *sm_count = p.multiProcessorCount;
  if (cc_major) *cc_major = p.major;
  if (cc_minor) *cc_minor = p.minor;
  if (total_mem) *total_mem = p.totalGlobalMem;
  return TL_OK;
}

const char* tl_error_string(int status) {
  switch (status) {
    case TL_OK: return "success";
    case TL_ERR_INVALID_ARG: return "invalid argument (size, pointer or op code)";
    case TL_ERR_ALIGNMENT: return "pointer or leading dimension violates required alignment";
    case TL_ERR_JIT: return "NVRTC compile or module load failed (see tl_jit_log)";
    case TL_ERR_NO_NCCL: return "libnccl.so.2 could not be loaded";
    case TL_ERR_NCCL: return "NCCL call failed";
    case TL_ERR_TIMEOUT: return "bounded wait timed out";
    case TL_ERR_NOT_INIT: return "tl_init was not called for this device";
    case TL_ERR_UNSUPPORTED: return "unsupported shape or layout for this kernel";
    default: return cudaGetErrorString((cudaError_t)status);
  }
}

void* tl_default_stream(void) { return (void*)tl::stream_or_default(nullptr); }

// ---------------------------------------------------------------- memory ---
int tl_malloc(void** ptr, size_t bytes, void* stream) {
  if (!ptr) return TL_ERR_INVALID_ARG;
  *ptr = nullptr;
  if (bytes == 0) bytes = 256;
  TL_CUDA_TRY(cudaMallocAsync(ptr, bytes, tl::stream_or_default(stream)));
  return TL_OK;
}

int tl_free(void* ptr, void* stream) {
  if (!ptr) return TL_OK;
  TL_CUDA_TRY(cudaFreeAsync(ptr, tl::stream_or_default(stream)));
  return TL_OK;
}

int tl_host_alloc(void** ptr, size_t bytes) {
  TL_CUDA_TRY(cudaHostAlloc(ptr, bytes ? bytes : 16, cudaHostAllocDefault));
  return TL_OK;
}

int tl_host_free(void* ptr) {
  TL_CUDA_TRY(cudaFreeHost(ptr));
  return TL_OK;
}

int tl_memcpy_h2d(void* dst, const void* src, size_t bytes, void* stream) {
  if (!bytes) return TL_OK;
  TL_CUDA_TRY(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, tl::stream_or_default(stream)));
  return TL_OK;
}

int tl_memcpy_d2h(void* dst, const void* src, size_t bytes, void* stream) {
  if (!bytes) return TL_OK;
  TL_CUDA_TRY(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, tl::stream_or_default(stream)));
  return TL_OK;
}

int tl_memcpy_d2d(void* dst, const void* src, size_t bytes, void* stream) {
  if (!bytes || dst == src) return TL_OK;
  TL_CUDA_TRY(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, tl::stream_or_default(stream)));
  return TL_OK;
}

int tl_memset(void* dst, int value, size_t bytes, void* stream) {
  if (!bytes) return TL_OK;
  TL_CUDA_TRY(cudaMemsetAsync(dst, value, bytes, tl::stream_or_default(stream)));
  return TL_OK;
}

// ------------------------------------------------------- streams, events ---
int tl_stream_create(void** stream) {
  cudaStream_t s;
  TL_CUDA_TRY(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
  *stream = (void*)s;
  return TL_OK;
}
int tl_stream_create_priority(void** stream, int urgent) {
  if (!stream) return TL_ERR_INVALID_ARG;
  int least = 0, greatest = 0;
  TL_CUDA_TRY(cudaDeviceGetStreamPriorityRange(&least, &greatest));
  cudaStream_t s;
  TL_CUDA_TRY(cudaStreamCreateWithPriority(&s, cudaStreamNonBlocking, urgent ? greatest : least));
  *stream = s;
  return TL_OK;
}

int tl_stream_destroy(void* stream) {
  TL_CUDA_TRY(cudaStreamDestroy((cudaStream_t)stream));
  return TL_OK;
}
int tl_stream_sync(void* stream) {
  TL_CUDA_TRY(cudaStreamSynchronize(tl::stream_or_default(stream)));
  return TL_OK;
}
int tl_device_sync(void) {
  TL_CUDA_TRY(cudaDeviceSynchronize());
  return TL_OK;
}
int tl_event_create(void** event) {
  cudaEvent_t e;
  TL_CUDA_TRY(cudaEventCreate(&e));
  *event = (void*)e;
  return TL_OK;
}
int tl_event_destroy(void* event) {
  TL_CUDA_TRY(cudaEventDestroy((cudaEvent_t)event));
  return TL_OK;
}
int tl_event_record(void* event, void* stream) {
  TL_CUDA_TRY(cudaEventRecord((cudaEvent_t)event, tl::stream_or_default(stream)));
  return TL_OK;
}
int tl_event_elapsed_ms(void* start, void* end, float* ms) {
  TL_CUDA_TRY(cudaEventElapsedTime(ms, (cudaEvent_t)start, (cudaEvent_t)end));
  return TL_OK;
}
int tl_stream_wait_event(void* stream, void* event) {
  TL_CUDA_TRY(cudaStreamWaitEvent(tl::stream_or_default(stream), (cudaEvent_t)event, 0));
  return TL_OK;
}

// ---------------------------------------------------------------- graphs ---
int tl_graph_begin(void* stream) {
  TL_CUDA_TRY(cudaStreamBeginCapture(tl::stream_or_default(stream), cudaStreamCaptureModeThreadLocal));
  return TL_OK;
}
// kernel nodes of the last captured graph, and how many of them carry a
// priority other than the default (captured from a priority stream)
static thread_local int t_graph_kernels = 0, t_graph_prioritised = 0;

int tl_graph_end(void* stream, void** graph_exec) {
  cudaGraph_t g = nullptr;
  TL_CUDA_TRY(cudaStreamEndCapture(tl::stream_or_default(stream), &g));
  t_graph_kernels = t_graph_prioritised = 0;
  size_t n = 0;
  if (cudaGraphGetNodes(g, nullptr, &n) == cudaSuccess && n > 0) {
    std::vector<cudaGraphNode_t> nodes(n);
    if (cudaGraphGetNodes(g, nodes.data(), &n) == cudaSuccess) {
      for (size_t i = 0; i < n; ++i) {
        cudaGraphNodeType ty;
        if (cudaGraphNodeGetType(nodes[i], &ty) != cudaSuccess || ty != cudaGraphNodeTypeKernel) continue;
        ++t_graph_kernels;
        cudaLaunchAttributeValue v{};
        if (cudaGraphKernelNodeGetAttribute(nodes[i], cudaLaunchAttributePriority, &v) == cudaSuccess &&
            v.priority != 0)
          ++t_graph_prioritised;
      }
    }
  }
  cudaGetLastError();
  cudaGraphExec_t ex = nullptr;
  // node priorities as captured: the gradient all-reduce's kernels keep the
  // communication stream's priority inside the graph (by default a graph runs
  // every node at the priority of the stream it is launched into)
  cudaError_t e = cudaGraphInstantiate(&ex, g, (unsigned long long)cudaGraphInstantiateFlagUseNodePriority);
  cudaGraphDestroy(g);
  if (e != cudaSuccess) return (int)e;
  *graph_exec = (void*)ex;
  return TL_OK;
}
int tl_graph_launch(void* graph_exec, void* stream) {
  TL_CUDA_TRY(cudaGraphLaunch((cudaGraphExec_t)graph_exec, tl::stream_or_default(stream)));
  return TL_OK;
}
int tl_graph_destroy(void* graph_exec) {
  TL_CUDA_TRY(cudaGraphExecDestroy((cudaGraphExec_t)graph_exec));
  return TL_OK;
}

int tl_graph_last_stats(int* kernel_nodes, int* prioritised_nodes) {
  if (kernel_nodes) *kernel_nodes = t_graph_kernels;
  if (prioritised_nodes) *prioritised_nodes = t_graph_prioritised;
  return TL_OK;
}

int tl_launch_counter(uint64_t* count, int reset) {
  if (count) *count = t_launches;
  if (reset) t_launches = 0;
  return TL_OK;
}

}  // extern "C"

// =========================================================== region JIT ===
namespace {

typedef CUresult (*PFN_ModuleLoadData)(CUmodule*, const void*);
typedef CUresult (*PFN_ModuleGetFunction)(CUfunction*, CUmodule, const char*);
typedef CUresult (*PFN_LaunchKernel)(CUfunction, unsigned, unsigned, unsigned, unsigned, unsigned,
                                     unsigned, unsigned, CUstream, void**, void**);

struct DriverApi {
  bool ok = false;
  PFN_ModuleLoadData load = nullptr;
  PFN_ModuleGetFunction getfn = nullptr;
  PFN_LaunchKernel launch = nullptr;
};

DriverApi g_drv;
std::once_flag g_drv_once;

void load_driver() {
  std::call_once(g_drv_once, [] {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuModuleLoadData", &p, cudaEnableDefault, &q) != cudaSuccess) return;
    g_drv.load = (PFN_ModuleLoadData)p;
    if (cudaGetDriverEntryPoint("cuModuleGetFunction", &p, cudaEnableDefault, &q) != cudaSuccess) return;
    g_drv.getfn = (PFN_ModuleGetFunction)p;
    if (cudaGetDriverEntryPoint("cuLaunchKernel", &p, cudaEnableDefault, &q) != cudaSuccess) return;
    g_drv.launch = (PFN_LaunchKernel)p;
    g_drv.ok = g_drv.load && g_drv.getfn && g_drv.launch;
  });
}

std::mutex g_jit_mu;
std::unordered_map<std::string, CUfunction> g_jit_cache;  // "<device>:<key>" -> function

bool read_file(const std::string& path, std::string* out) {
  std::ifstream f(path, std::ios::binary);
  if (!f) return false;
  std::ostringstream ss;
  ss << f.rdbuf();
  *out = ss.str();
  return !out->empty();
}

void write_file_atomic(const std::string& path, const std::string& data) {
  std::string tmp = path + ".tmp." + std::to_string((unsigned long long)std::hash<std::thread::id>{}(std::this_thread::get_id()));
  {
    std::ofstream f(tmp, std::ios::binary);
    if (!f) return;
    f.write(data.data(), (std::streamsize)data.size());
  }
  std::rename(tmp.c_str(), path.c_str());
}

int nvrtc_compile(const char* source, std::string* cubin) {
  nvrtcProgram prog;
  if (nvrtcCreateProgram(&prog, source, "tl_region.cu", 0, nullptr, nullptr) != NVRTC_SUCCESS)
    return TL_ERR_JIT;
  const char* opts[] = {"--gpu-architecture=sm_100a", "--std=c++17", "-default-device",
                        "--extra-device-vectorization", "-lineinfo"};
  nvrtcResult r = nvrtcCompileProgram(prog, (int)(sizeof(opts) / sizeof(opts[0])), opts);
  size_t log_size = 0;
  nvrtcGetProgramLogSize(prog, &log_size);
  std::string log(log_size, '\0');
  if (log_size) nvrtcGetProgramLog(prog, &log[0]);
  t_jit_log = log;
  if (r != NVRTC_SUCCESS) {
    nvrtcDestroyProgram(&prog);
    return TL_ERR_JIT;
  }
  size_t n = 0;
  nvrtcGetCUBINSize(prog, &n);
  cubin->resize(n);
  nvrtcGetCUBIN(prog, &(*cubin)[0]);
  nvrtcDestroyProgram(&prog);
  return TL_OK;
}

}  // namespace

extern "C" {

const char* tl_jit_log(void) { return t_jit_log.c_str(); }

int tl_jit_compile(const char* source, const char* kernel_name, const char* key,
                   const char* cache_dir, void** function) {
  if (!source || !kernel_name || !key || !function) return TL_ERR_INVALID_ARG;
  load_driver();
  if (!g_drv.ok) return TL_ERR_JIT;
  int dev = current_device();
  std::string ck = std::to_string(dev) + ":" + key;
  {
    std::lock_guard<std::mutex> lk(g_jit_mu);
    auto it = g_jit_cache.find(ck);
    if (it != g_jit_cache.end()) {
      *function = (void*)it->second;
      return TL_OK;
    }
  }
  std::string cubin;
  std::string path;
  if (cache_dir && *cache_dir) path = std::string(cache_dir) + "/" + key + ".cubin";
  if (path.empty() || !read_file(path, &cubin)) {
    TL_TRY(nvrtc_compile(source, &cubin));
    if (!path.empty()) write_file_atomic(path, cubin);
  }
  CUmodule mod;
  if (g_drv.load(&mod, cubin.data()) != CUDA_SUCCESS) return TL_ERR_JIT;
  CUfunction fn;
  if (g_drv.getfn(&fn, mod, kernel_name) != CUDA_SUCCESS) return TL_ERR_JIT;
  {
    std::lock_guard<std::mutex> lk(g_jit_mu);
    g_jit_cache[ck] = fn;
  }
  *function = (void*)fn;
  return TL_OK;
}

int tl_jit_launch(void* function, unsigned grid, unsigned block, unsigned smem, void** args,
                  void* stream) {
  if (!function || !grid || !block) return TL_ERR_INVALID_ARG;
  load_driver();
  if (!g_drv.ok) return TL_ERR_JIT;
  CUresult r = g_drv.launch((CUfunction)function, grid, 1, 1, block, 1, 1, smem,
                            (CUstream)tl::stream_or_default(stream), args, nullptr);
  ++t_launches;
  if (r != CUDA_SUCCESS) return TL_ERR_JIT;
  return TL_OK;
}

}  // extern "C"

// ================================================================ NCCL ====
namespace {

struct NcclApi {
  bool ok = false;
  ncclResult_t (*getUniqueId)(ncclUniqueId*);
  ncclResult_t (*commInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*);
  ncclResult_t (*allReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                            cudaStream_t);
  ncclResult_t (*commGetAsyncError)(ncclComm_t, ncclResult_t*);
  ncclResult_t (*commDestroy)(ncclComm_t);
  ncclResult_t (*commAbort)(ncclComm_t);
  ncclResult_t (*commFinalize)(ncclComm_t);
};

NcclApi g_nccl;
std::once_flag g_nccl_once;

void load_nccl() {
  std::call_once(g_nccl_once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_LOCAL);
    if (!h) return;
#define TL_SYM(field, name)                                   \
  g_nccl.field = (decltype(g_nccl.field))dlsym(h, name);       \
  if (!g_nccl.field) return;
    TL_SYM(getUniqueId, "ncclGetUniqueId");
    TL_SYM(commInitRankConfig, "ncclCommInitRankConfig");
    TL_SYM(allReduce, "ncclAllReduce");
    TL_SYM(commGetAsyncError, "ncclCommGetAsyncError");
    TL_SYM(commDestroy, "ncclCommDestroy");
    TL_SYM(commAbort, "ncclCommAbort");
    TL_SYM(commFinalize, "ncclCommFinalize");
#undef TL_SYM
    g_nccl.ok = true;
  });
}

// Poll a non-blocking communicator until it leaves ncclInProgress.
int nccl_settle(ncclComm_t comm, int timeout_ms) {
  auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    ncclResult_t st = ncclSuccess;
    if (g_nccl.commGetAsyncError(comm, &st) != ncclSuccess) return TL_ERR_NCCL;
    if (st == ncclSuccess) return TL_OK;
    if (st != ncclInProgress) return TL_ERR_NCCL;
    auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(
                  std::chrono::steady_clock::now() - t0).count();
    if (timeout_ms >= 0 && ms > timeout_ms) return TL_ERR_TIMEOUT;
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

}  // namespace

extern "C" {

int tl_nccl_unique_id(unsigned char id[128]) {
  load_nccl();
  if (!g_nccl.ok) return TL_ERR_NO_NCCL;
  ncclUniqueId u;
  if (g_nccl.getUniqueId(&u) != ncclSuccess) return TL_ERR_NCCL;
  static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId size");
  std::memcpy(id, &u, 128);
  return TL_OK;
}

int tl_nccl_comm_init(void** comm, int nranks, const unsigned char id[128], int rank, int timeout_ms) {
  load_nccl();
  if (!g_nccl.ok) return TL_ERR_NO_NCCL;
  ncclUniqueId u;
  std::memcpy(&u, id, 128);
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  ncclComm_t c = nullptr;
  ncclResult_t r = g_nccl.commInitRankConfig(&c, nranks, u, rank, &cfg);
  if (r != ncclSuccess && r != ncclInProgress) return TL_ERR_NCCL;
  int s = nccl_settle(c, timeout_ms);
  if (s != TL_OK) {
    g_nccl.commAbort(c);
    return s;
  }
  *comm = (void*)c;
  return TL_OK;
}

int tl_nccl_allreduce_sum(void* comm, float* buf, size_t count, void* stream) {
  if (!g_nccl.ok) return TL_ERR_NO_NCCL;
  ncclResult_t r = g_nccl.allReduce(buf, buf, count, ncclFloat32, ncclSum, (ncclComm_t)comm,
                                    tl::stream_or_default(stream));
  if (r == ncclInProgress) return nccl_settle((ncclComm_t)comm, 60000);  // enqueue finishing
  if (r != ncclSuccess) return TL_ERR_NCCL;
  return TL_OK;
}

int tl_nccl_wait(void* comm, void* stream, int timeout_ms) {
  if (!g_nccl.ok) return TL_ERR_NO_NCCL;
  auto t0 = std::chrono::steady_clock::now();
  cudaStream_t s = tl::stream_or_default(stream);
  for (;;) {
    ncclResult_t st = ncclSuccess;
    if (g_nccl.commGetAsyncError((ncclComm_t)comm, &st) != ncclSuccess) return TL_ERR_NCCL;
    if (st != ncclSuccess && st != ncclInProgress) return TL_ERR_NCCL;
    cudaError_t q = cudaStreamQuery(s);
    if (q == cudaSuccess && st == ncclSuccess) return TL_OK;
    if (q != cudaSuccess && q != cudaErrorNotReady) return (int)q;
    auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(
                  std::chrono::steady_clock::now() - t0).count();
    if (timeout_ms >= 0 && ms > timeout_ms) {
      g_nccl.commAbort((ncclComm_t)comm);
      return TL_ERR_TIMEOUT;
    }
    std::this_thread::sleep_for(std::chrono::microseconds(20));
  }
}

int tl_nccl_comm_destroy(void* comm) {
  if (!g_nccl.ok) return TL_ERR_NO_NCCL;
  ncclComm_t c = (ncclComm_t)comm;
  ncclResult_t r = g_nccl.commFinalize(c);
  if (r == ncclInProgress) {
    if (nccl_settle(c, 30000) != TL_OK) {
      g_nccl.commAbort(c);
      return TL_ERR_TIMEOUT;
    }
  } else if (r != ncclSuccess) {
    g_nccl.commAbort(c);
    return TL_ERR_NCCL;
  }
  g_nccl.commDestroy(c);
  return TL_OK;
}

int tl_nccl_comm_abort(void* comm) {
  if (!g_nccl.ok) return TL_ERR_NO_NCCL;
  g_nccl.commAbort((ncclComm_t)comm);
  return TL_OK;
}

}  // extern "C"
