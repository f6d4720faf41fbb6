// zg_noalloc.cu -- a replay entry point that allocates nothing.
//
// zg_replay needs scratch (the candidates' factors) and takes it from a
// workspace the caller allocates.  Some callers cannot do that where they run
// the replay: a host that hands the GPU library one memory pool at start-up
// and forbids any later cudaMalloc (embedded and certified deployments,
// schedulers that account for every device byte up front), or code that must
// not call an allocator because an allocation may synchronise the device or
// take a lock on a latency-critical thread.  zg_replay_noalloc serves them:
// it runs exactly zg_replay, with the scratch taken from a buffer compiled
// into this library.
//
// The buffer is a file-scope __device__ array of kNoAllocScratchBytes.  Every
// GPU that loads this library's device code holds those bytes until the
// process exits.  In host code the array's name is only a host-side handle,
// not a device address, so the device address is looked up with
// cudaGetSymbolAddress once per device (on the first call made with that
// device current) and cached for the process (a cudaDeviceReset between calls
// would leave the cached address stale: not supported).  This file is its own
// module; under lazy module loading the lookup loads it, so the first call on
// a device is the one that takes the 16 MiB.
#include <mutex>

#include "zg_common.cuh"

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;  // 16 MiB
static __device__ __align__(256) unsigned char zg_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
void* g_scratch_addr[kMaxDevices] = {};

}  // namespace

extern "C" int zg_replay_noalloc(const float* shaped, const uint32_t* keys, int group, int P, int layout,
                                 int64_t rows, int64_t cols, int rank, float inv_sqrt_rank, int dtype, float* out,
                                 void* stream) {
    const size_t need = zg_replay_workspace_size(P, layout, rows, cols, rank, dtype);
    if (need == 0)
        return zg::fail(ZG_ERR_INVALID, "zg_replay_noalloc: bad sizes, layout or dtype");
    if (need > kNoAllocScratchBytes)
        return zg::fail(ZG_ERR_WORKSPACE,
                        "zg_replay_noalloc: this replay needs %zu bytes of scratch but the library holds %zu; "
                        "call zg_replay with a workspace of zg_replay_workspace_size() bytes instead",
                        need, kNoAllocScratchBytes);
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
        return zg::fail(ZG_ERR_CUDA, "zg_replay_noalloc: no usable current device");
    void* scratch = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_scratch_mu);
        if (!g_scratch_addr[dev]) {
            void* p = nullptr;
            const cudaError_t e = cudaGetSymbolAddress(&p, zg_noalloc_scratch);
            if (e != cudaSuccess || !p)
                return zg::fail(ZG_ERR_CUDA, "zg_replay_noalloc: cudaGetSymbolAddress failed on device %d: %s",
                                dev, cudaGetErrorString(e));
            g_scratch_addr[dev] = p;
        }
        scratch = g_scratch_addr[dev];
    }
    // Every scratch byte the replay reads is written earlier in the same call,
    // so nothing needs clearing between calls.
    return zg_replay(shaped, keys, group, P, layout, rows, cols, rank, inv_sqrt_rank, dtype, out, scratch,
                     kNoAllocScratchBytes, stream);
}
