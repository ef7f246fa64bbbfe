// Device memory guard: exact accounting for every cudaMalloc the library makes,
// plus a measured gate on device memory.
//
// Same contract as the reference guard (src/memory_guard.cpp, declared in
// include/aero/memory_guard.hpp):
//   * try_reserve(bytes, class) refuses a reservation that would push the
//     committed total past the budget, after giving a registered evictor one
//     chance to free cache bytes (src/memory_guard.cpp:155-184); budget 0 means
//     unbounded. release() never goes below zero (:186-190).
//   * admit_plan refuses a whole load up front (:192-213).
//   * LoadGate reserves a load chunk by chunk, treats a final partial chunk as
//     completion rather than failure, and can pause between chunks and check
//     the measured footprint (:314-378).
//   * A monitor thread samples the measured footprint and calls the breach
//     handler once (:252-286).
// What changes for the GPU: the measured footprint is device memory in use on
// this process's device as cudaMemGetInfo reports it, minus the usage seen when
// the guard first measured (other tenants of a shared GPU are not charged to
// this process). The default breach handler reports and marks the guard as
// exceeded; it does not terminate the process (the reference _exit(87)s, which
// on a shared device would let another tenant's allocation kill this process).
#include <cuda_runtime.h>

#include <atomic>
#include <chrono>
#include <cstdio>
#include <functional>
#include <mutex>
#include <string>
#include <thread>

#include "internal.h"

namespace aero {

std::string fmt_bytes(size_t b) {
    static const char* u[] = {"B", "KiB", "MiB", "GiB", "TiB"};
    double v = (double)b;
    int i = 0;
    while (v >= 1024.0 && i < 4) {
        v /= 1024.0;
        ++i;
    }
    char buf[64];
    std::snprintf(buf, sizeof(buf), "%.2f %s", v, u[i]);
    return buf;
}

namespace {

struct Guard {
    std::mutex mu;
    size_t budget = 0;
    size_t committed[kMemClassCount] = {};
    std::function<size_t(size_t)> evictor;
    // test hook: refuse the n-th upcoming guarded allocation (1 = the next one)
    long fail_countdown = 0;
    // measured footprint baseline
    bool have_base = false;
    size_t base_used = 0;
    int device = 0;
    std::atomic<bool> stop{false}, exceeded{false};
    std::atomic<size_t> peak{0}, last{0};
    std::thread monitor;
    std::function<void(size_t, size_t)> on_breach;

    size_t total_locked() const {
        size_t t = 0;
        for (size_t v : committed) t += v;
        return t;
    }
};

Guard& G() {
    static Guard* g = new Guard();  // outlives every handle; never destroyed
    return *g;
}

size_t device_used(int device) {
    int prev = 0;
    cudaGetDevice(&prev);
    if (prev != device) cudaSetDevice(device);
    size_t free_b = 0, total_b = 0;
    const cudaError_t e = cudaMemGetInfo(&free_b, &total_b);
    if (prev != device) cudaSetDevice(prev);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return total_b - free_b;
}

}  // namespace

bool guard_try_reserve(size_t bytes, int cls) {
    Guard& g = G();
    std::function<size_t(size_t)> ev;
    {
        std::lock_guard<std::mutex> lk(g.mu);
        if (g.budget == 0 || g.total_locked() + bytes <= g.budget) {
            g.committed[cls] += bytes;
            return true;
        }
        ev = g.evictor;
    }
    if (ev) {
        ev(bytes);
        std::lock_guard<std::mutex> lk(g.mu);
        if (g.total_locked() + bytes <= g.budget) {
            g.committed[cls] += bytes;
            return true;
        }
    }
    return false;
}

void guard_release(size_t bytes, int cls) {
    Guard& g = G();
    std::lock_guard<std::mutex> lk(g.mu);
    size_t& s = g.committed[cls];
    s = bytes > s ? 0 : s - bytes;
}

cudaError_t guarded_malloc(void** p, size_t bytes, int cls) {
    *p = nullptr;
    {
        Guard& g = G();
        std::lock_guard<std::mutex> lk(g.mu);
        if (g.fail_countdown > 0 && --g.fail_countdown == 0) return cudaErrorMemoryAllocation;
    }
    if (!guard_try_reserve(bytes, cls)) return cudaErrorMemoryAllocation;
    const cudaError_t e = cudaMalloc(p, bytes);
    if (e != cudaSuccess) {
        guard_release(bytes, cls);
        *p = nullptr;
    }
    return e;
}

void guarded_free(void* p, size_t bytes, int cls) {
    if (!p) return;
    cudaFree(p);
    guard_release(bytes, cls);
}

}  // namespace aero

using aero::G;

extern "C" {

void aero_cuda_guard_set_budget(size_t bytes) {
    std::lock_guard<std::mutex> lk(G().mu);
    G().budget = bytes;
}
size_t aero_cuda_guard_budget(void) {
    std::lock_guard<std::mutex> lk(G().mu);
    return G().budget;
}
size_t aero_cuda_guard_committed(int cls) {
    std::lock_guard<std::mutex> lk(G().mu);
    if (cls < 0) return G().total_locked();
    if (cls >= aero::kMemClassCount) return 0;
    return G().committed[cls];
}
size_t aero_cuda_guard_headroom(void) {
    std::lock_guard<std::mutex> lk(G().mu);
    const size_t t = G().total_locked();
    return G().budget > t ? G().budget - t : 0;
}
int aero_cuda_guard_try_reserve(size_t bytes, int cls) {
    if (cls < 0 || cls >= aero::kMemClassCount) return 0;
    return aero::guard_try_reserve(bytes, cls) ? 1 : 0;
}
void aero_cuda_guard_release(size_t bytes, int cls) {
    if (cls < 0 || cls >= aero::kMemClassCount) return;
    aero::guard_release(bytes, cls);
}
int aero_cuda_guard_admit_plan(size_t planned, char* why, int why_len) {
    std::lock_guard<std::mutex> lk(G().mu);
    std::string w;
    int ok = 1;
    if (G().budget != 0) {
        const size_t t = G().total_locked();
        if (planned > G().budget) {
            w = "planned footprint " + aero::fmt_bytes(planned) + " exceeds the device budget " +
                aero::fmt_bytes(G().budget);
            ok = 0;
        } else if (t + planned > G().budget) {
            w = "already committed " + aero::fmt_bytes(t) + "; plan needs " + aero::fmt_bytes(planned) +
                " but budget is " + aero::fmt_bytes(G().budget);
            ok = 0;
        }
    }
    if (why && why_len > 0) std::snprintf(why, (size_t)why_len, "%s", w.c_str());
    return ok;
}
// Evictor: a C callback returning the bytes it freed; NULL clears it.
typedef size_t (*aero_cuda_evict_fn)(void* ctx, size_t need);
void aero_cuda_guard_set_evictor(aero_cuda_evict_fn fn, void* ctx) {
    std::lock_guard<std::mutex> lk(G().mu);
    if (fn)
        G().evictor = [fn, ctx](size_t need) { return fn(ctx, need); };
    else
        G().evictor = nullptr;
}
// Host-side fault injection: the n-th guarded allocation from now is refused.
void aero_cuda_guard_fail_nth_alloc(long n) {
    std::lock_guard<std::mutex> lk(G().mu);
    G().fail_countdown = n;
}

// Measured footprint: device bytes in use now minus those in use when first
// measured on this device.
size_t aero_cuda_guard_own_footprint(int device) {
    const size_t used = aero::device_used(device);
    std::lock_guard<std::mutex> lk(G().mu);
    if (!G().have_base || G().device != device) {
        G().have_base = true;
        G().device = device;
        G().base_used = used;
    }
    return used > G().base_used ? used - G().base_used : 0;
}
size_t aero_cuda_guard_device_free(int device) {
    int prev = 0;
    cudaGetDevice(&prev);
    if (prev != device) cudaSetDevice(device);
    size_t f = 0, t = 0;
    if (cudaMemGetInfo(&f, &t) != cudaSuccess) {
        cudaGetLastError();
        f = 0;
    }
    if (prev != device) cudaSetDevice(prev);
    return f;
}
int aero_cuda_guard_preflight(int device, size_t headroom) {
    size_t budget;
    {
        std::lock_guard<std::mutex> lk(G().mu);
        budget = G().budget;
    }
    if (budget == 0) return 1;
    const size_t avail = aero_cuda_guard_device_free(device);
    return avail >= budget + headroom ? 1 : 0;
}

typedef void (*aero_cuda_breach_fn)(void* ctx, size_t footprint, size_t budget);
void aero_cuda_guard_set_on_breach(aero_cuda_breach_fn fn, void* ctx) {
    std::lock_guard<std::mutex> lk(G().mu);
    if (fn)
        G().on_breach = [fn, ctx](size_t f, size_t b) { fn(ctx, f, b); };
    else
        G().on_breach = nullptr;
}
int aero_cuda_guard_exceeded(void) { return G().exceeded.load() ? 1 : 0; }
size_t aero_cuda_guard_peak_footprint(void) { return G().peak.load(); }
void aero_cuda_guard_reset_exceeded(void) { G().exceeded.store(false); }

void aero_cuda_guard_stop_monitor(void) {
    G().stop.store(true);
    if (G().monitor.joinable()) G().monitor.join();
}
void aero_cuda_guard_start_monitor(int device, unsigned interval_ms) {
    if (G().monitor.joinable()) return;
    if (interval_ms == 0) interval_ms = 50;
    G().stop.store(false);
    aero_cuda_guard_own_footprint(device);  // establish the baseline on this thread
    G().monitor = std::thread([device, interval_ms]() {
        while (!G().stop.load()) {
            const size_t fp = aero_cuda_guard_own_footprint(device);
            G().last.store(fp);
            size_t prev = G().peak.load();
            while (fp > prev && !G().peak.compare_exchange_weak(prev, fp)) {
            }
            size_t budget;
            std::function<void(size_t, size_t)> fn;
            {
                std::lock_guard<std::mutex> lk(G().mu);
                budget = G().budget;
                fn = G().on_breach;
            }
            if (budget > 0 && fp > budget) {
                G().exceeded.store(true);
                if (fn)
                    fn(fp, budget);
                else
                    std::fprintf(stderr, "[aero-b200] device footprint %s exceeds budget %s\n",
                                 aero::fmt_bytes(fp).c_str(), aero::fmt_bytes(budget).c_str());
                return;
            }
            std::this_thread::sleep_for(std::chrono::milliseconds(interval_ms));
        }
    });
}

// ---- LoadGate ------------------------------------------------------------
struct aero_cuda_loadgate {
    size_t planned = 0, taken = 0, reserved = 0;
    unsigned pause_ms = 0;
    int device = 0;
    int ok = 1, done = 0;
    std::string reason;
};

void* aero_cuda_loadgate_open(size_t planned, int device) {
    auto* g = new aero_cuda_loadgate();
    g->planned = planned;
    g->device = device;
    char why[256] = {0};
    if (!aero_cuda_guard_admit_plan(planned, why, sizeof(why))) {
        g->ok = 0;
        g->reason = why;
    }
    return g;
}
void aero_cuda_loadgate_close(void* h) { delete static_cast<aero_cuda_loadgate*>(h); }
void aero_cuda_loadgate_set_pause_ms(void* h, unsigned ms) { static_cast<aero_cuda_loadgate*>(h)->pause_ms = ms; }

static int loadgate_check_measured(aero_cuda_loadgate* g) {
    if (!g->ok) return 0;
    const size_t fp = aero_cuda_guard_own_footprint(g->device);
    const size_t b = aero_cuda_guard_budget();
    if (b > 0 && fp > b) {
        g->ok = 0;
        g->reason = "measured device footprint " + aero::fmt_bytes(fp) + " exceeded the budget mid-load; load stopped";
        return 0;
    }
    return 1;
}

int aero_cuda_loadgate_next_chunk(void* h, size_t chunk, int cls) {
    auto* g = static_cast<aero_cuda_loadgate*>(h);
    if (!g->ok || g->done) return 0;
    if (g->taken >= g->planned || g->taken + chunk > g->planned) {
        g->done = 1;  // the admitted plan is satisfied: completion, not a failure
        return 0;
    }
    if (cls < 0 || cls >= aero::kMemClassCount || !aero::guard_try_reserve(chunk, cls)) {
        g->ok = 0;
        g->reason = "next chunk of " + aero::fmt_bytes(chunk) + " would exceed the device budget; load stopped";
        return 0;
    }
    g->taken += chunk;
    g->reserved += chunk;
    if (g->pause_ms > 0) {
        std::this_thread::sleep_for(std::chrono::milliseconds(g->pause_ms));
        if (!loadgate_check_measured(g)) return 0;
    }
    return 1;
}
int aero_cuda_loadgate_pause_and_check(void* h) {
    auto* g = static_cast<aero_cuda_loadgate*>(h);
    if (!g->ok) return 0;
    if (g->pause_ms > 0)
        std::this_thread::sleep_for(std::chrono::milliseconds(g->pause_ms));
    else
        std::this_thread::yield();
    return loadgate_check_measured(g);
}
int aero_cuda_loadgate_ok(void* h) { return static_cast<aero_cuda_loadgate*>(h)->ok; }
int aero_cuda_loadgate_done(void* h) { return static_cast<aero_cuda_loadgate*>(h)->done; }
size_t aero_cuda_loadgate_taken(void* h) { return static_cast<aero_cuda_loadgate*>(h)->taken; }
size_t aero_cuda_loadgate_reserved(void* h) { return static_cast<aero_cuda_loadgate*>(h)->reserved; }
size_t aero_cuda_loadgate_remaining(void* h) {
    auto* g = static_cast<aero_cuda_loadgate*>(h);
    return g->planned > g->taken ? g->planned - g->taken : 0;
}
int aero_cuda_loadgate_reason(void* h, char* buf, int len) {
    auto* g = static_cast<aero_cuda_loadgate*>(h);
    if (buf && len > 0) std::snprintf(buf, (size_t)len, "%s", g->reason.c_str());
    return (int)g->reason.size();
}

}  // extern "C"
