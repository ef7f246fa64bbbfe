// aero_cuda_dispatch_noalloc: the expert dispatch with no device allocation.
//
// Who needs it: callers that may not allocate device memory at the moment they
// route tokens. Two common cases: a process whose device budget is already
// fully committed (the memory guard refuses any further cudaMalloc, yet
// routing must still run), and a pipeline that cannot afford cudaMalloc's
// implicit device-wide synchronisation between its kernels. aero_cuda_dispatch
// takes its scratch from the guard for every call; this variant takes it from
// one fixed array instead.
//
// The scratch is `g_noalloc_scratch` below, a file-scope __device__ array of
// kNoAllocScratchBytes (2 MiB). Every GPU that loads this library holds that
// array until the process exits. Host code may not use the array's name as a
// device address (on the host it names a stand-in object, not device memory),
// so the first call on each device, with that device current, asks the runtime
// for the real address with cudaGetSymbolAddress and caches it. That first call
// is the set-up step: make it before any stream capture.
//
// All calls on a device share the one array, and it keeps whatever the last
// call left in it. The error flag is cleared at the start of every call; the
// histogram and the other intermediate arrays are fully rewritten by each call
// before they are read. Two calls whose work overlaps on the GPU (for example
// on two streams at once) race on the array and produce wrong results: order
// them on one stream, or finish one before starting the next.
#include <cuda_runtime.h>

#include <cstdio>
#include <mutex>
#include <string>

#include "../../include/aero_cuda_moe.h"
#include "internal.h"

namespace aero {
namespace {

constexpr int kNoAllocMaxPairs = 65536;   // T * k
constexpr int kNoAllocMaxExperts = 1024;  // n_expert
constexpr size_t kNoAllocScratchBytes = 2u << 20;
constexpr int kMaxDevices = 64;

// Layout of the array (byte offsets, 256-byte aligned regions).
constexpr size_t al256(size_t v) { return (v + 255) & ~(size_t)255; }
constexpr size_t kOffIdx = 0;                                                   // int32 expert ids, P
constexpr size_t kOffInv = kOffIdx + al256((size_t)kNoAllocMaxPairs * 4);       // int32, P
constexpr size_t kOffActE = kOffInv + al256((size_t)kNoAllocMaxPairs * 4);      // int32, E
constexpr size_t kOffActOff = kOffActE + al256((size_t)kNoAllocMaxExperts * 4); // int32, E + 1
constexpr size_t kOffNAct = kOffActOff + al256((size_t)(kNoAllocMaxExperts + 1) * 4);
constexpr size_t kOffFlag = kOffNAct + 256;                                     // int32 error flag
constexpr size_t kOffWork = kOffFlag + 256;                                     // per-chunk histograms
static_assert(kOffWork + (size_t)((kNoAllocMaxPairs + 255) / 256 + 1) * kNoAllocMaxExperts * 4 <= kNoAllocScratchBytes,
              "no-alloc scratch layout does not fit");

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_mu;
void* g_addr[kMaxDevices] = {};

// Device address of the array on the current device (set up on first use).
void* scratch_address(int device, std::string* why) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (g_addr[device]) return g_addr[device];
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p) {
        cudaGetLastError();
        *why = std::string("cudaGetSymbolAddress of the no-alloc scratch failed: ") + cudaGetErrorString(e);
        return nullptr;
    }
    g_addr[device] = p;
    return p;
}

// int64 expert ids -> int32, with a range check. An out-of-range id raises the
// flag and is replaced by 0 so the histogram stays in bounds.
__global__ void narrow_ids_kernel(const int64_t* __restrict__ idx, int P, int E, int32_t* __restrict__ out,
                                  int32_t* __restrict__ flag) {
    const int p = blockIdx.x * blockDim.x + threadIdx.x;
    if (p >= P) return;
    const int64_t v = idx[p];
    const bool ok = v >= 0 && v < E;
    out[p] = ok ? (int32_t)v : 0;
    if (!ok) atomicExch(flag, 1);
}

bool is_device_memory(const void* p) {
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged;
}

}  // namespace
}  // namespace aero

extern "C" int aero_cuda_dispatch_noalloc(const int64_t* idx, int T, int k, int n_expert, int32_t* offsets,
                                          int32_t* perm, void* stream) {
    using namespace aero;
    if (T < 0 || k <= 0 || n_expert <= 0) {
        set_free_error("T must be >= 0 and k, n_expert positive");
        return -1;
    }
    const int64_t P = (int64_t)T * k;
    if (P > kNoAllocMaxPairs || n_expert > kNoAllocMaxExperts) {
        char b[200];
        std::snprintf(b, sizeof(b),
                      "no-alloc dispatch handles at most %d (token, slot) pairs and %d experts; got %lld pairs, %d "
                      "experts (use aero_cuda_dispatch)",
                      kNoAllocMaxPairs, kNoAllocMaxExperts, (long long)P, n_expert);
        set_free_error(b);
        return -1;
    }
    if (!idx || !offsets || (P > 0 && !perm) || !is_device_memory(idx) || !is_device_memory(offsets) ||
        (P > 0 && !is_device_memory(perm))) {
        set_free_error("no-alloc dispatch needs device pointers for idx, offsets and perm");
        return -1;
    }
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        cudaGetLastError();
        set_free_error("no current CUDA device");
        return -1;
    }
    std::string why;
    char* base = static_cast<char*>(scratch_address(dev, &why));
    if (!base) {
        set_free_error(why);
        return -1;
    }
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    int32_t* flag = reinterpret_cast<int32_t*>(base + kOffFlag);
    int32_t* ids = reinterpret_cast<int32_t*>(base + kOffIdx);
    cudaError_t e = cudaMemsetAsync(flag, 0, sizeof(int32_t), st);
    if (e == cudaSuccess && P > 0) {
        narrow_ids_kernel<<<(unsigned)((P + 255) / 256), 256, 0, st>>>(idx, (int)P, n_expert, ids, flag);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess)
        e = launch_dispatch(ids, (int)P, n_expert, offsets, perm, reinterpret_cast<int32_t*>(base + kOffInv),
                            reinterpret_cast<int32_t*>(base + kOffActE), reinterpret_cast<int32_t*>(base + kOffActOff),
                            reinterpret_cast<int32_t*>(base + kOffNAct), base + kOffWork, st);
    int32_t host_flag = 0;
    if (e == cudaSuccess) e = cudaMemcpyAsync(&host_flag, flag, sizeof(int32_t), cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) {
        cudaGetLastError();
        set_free_error(std::string("no-alloc dispatch: ") + cudaGetErrorString(e));
        return -1;
    }
    if (host_flag) {
        set_free_error("expert index out of range");
        return -1;
    }
    return 0;
}

