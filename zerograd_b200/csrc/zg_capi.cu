// zg_capi.cu -- error state and version of the libzgb200 C ABI.
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "zg_common.cuh"

namespace zg {

static thread_local char g_last_error[1024] = "";

void set_error(const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
    va_end(ap);
}

int fail(int code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
    va_end(ap);
    return code;
}

int check_launch(const char* what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(ZG_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
    return ZG_OK;
}

// ---------------------------------------------------------------------------
// launch accounting / profiling
// ---------------------------------------------------------------------------
static std::atomic<int64_t> g_launches{0};
static std::mutex g_prof_mu;
static bool g_prof_on = false;
struct ProfRec {
    const char* name;
    cudaEvent_t start, stop;
};
static std::vector<ProfRec> g_prof;
static size_t g_prof_used = 0;

LaunchTimer::LaunchTimer(const char* name, cudaStream_t st) : stream(st) {
    g_launches.fetch_add(1, std::memory_order_relaxed);
    if (!g_prof_on) return;
    std::lock_guard<std::mutex> lk(g_prof_mu);
    if (!g_prof_on || g_prof_used >= g_prof.size()) return;
    slot = (int)g_prof_used++;
    g_prof[slot].name = name;
    cudaEventRecord(g_prof[slot].start, st);
}

LaunchTimer::~LaunchTimer() {
    if (slot >= 0) cudaEventRecord(g_prof[slot].stop, stream);
}

}  // namespace zg

extern "C" int64_t zg_launch_count(void) { return zg::g_launches.load(); }

extern "C" int zg_profile_begin(int max_records) {
    if (max_records < 1 || max_records > (1 << 20)) return zg::fail(ZG_ERR_INVALID, "zg_profile_begin: bad size");
    std::lock_guard<std::mutex> lk(zg::g_prof_mu);
    while ((int)zg::g_prof.size() < max_records) {
        zg::ProfRec r{nullptr, nullptr, nullptr};
        if (cudaEventCreate(&r.start) != cudaSuccess || cudaEventCreate(&r.stop) != cudaSuccess)
            return zg::fail(ZG_ERR_CUDA, "zg_profile_begin: cudaEventCreate failed");
        zg::g_prof.push_back(r);
    }
    zg::g_prof_used = 0;
    zg::g_prof_on = true;
    return ZG_OK;
}

extern "C" int zg_profile_end(void) {
    std::lock_guard<std::mutex> lk(zg::g_prof_mu);
    zg::g_prof_on = false;
    return ZG_OK;
}

extern "C" int zg_profile_summary(char* buf, size_t len) {
    std::lock_guard<std::mutex> lk(zg::g_prof_mu);
    std::map<std::string, std::pair<int, double>> agg;
    for (size_t i = 0; i < zg::g_prof_used; ++i) {
        auto& r = zg::g_prof[i];
        if (cudaEventSynchronize(r.stop) != cudaSuccess)
            return zg::fail(ZG_ERR_CUDA, "zg_profile_summary: event sync failed");
        float ms = 0.f;
        if (cudaEventElapsedTime(&ms, r.start, r.stop) != cudaSuccess)
            return zg::fail(ZG_ERR_CUDA, "zg_profile_summary: elapsed time failed");
        auto& e = agg[r.name];
        e.first += 1;
        e.second += ms;
    }
    std::string out;
    char line[256];
    for (auto& kv : agg) {
        snprintf(line, sizeof(line), "%s,%d,%.6f\n", kv.first.c_str(), kv.second.first, kv.second.second);
        out += line;
    }
    if (!buf || len == 0) return zg::fail(ZG_ERR_INVALID, "zg_profile_summary: no buffer");
    if (out.size() + 1 > len) return zg::fail(ZG_ERR_INVALID, "zg_profile_summary: buffer too small");
    memcpy(buf, out.c_str(), out.size() + 1);
    return ZG_OK;
}

extern "C" const char* zg_last_error(void) { return zg::g_last_error; }

extern "C" const char* zg_version(void) { return "zgb200 0.1 (sm_100a)"; }
