// Library-wide C ABI entry points: status strings, version, launch policy.
#include "kb_common.cuh"

#include <atomic>
#include <cstdlib>
#include <cstring>
#include <mutex>

namespace kb {

namespace {
int initial_pdl() {
    const char* v = std::getenv("KB_PDL");
    if (v && (std::strcmp(v, "0") == 0 || std::strcmp(v, "off") == 0)) return 0;
    return 1;
}
std::atomic<int> g_pdl{initial_pdl()};
}  // namespace

bool pdl_enabled() { return g_pdl.load(std::memory_order_relaxed) != 0; }

int device_sm_count() {
    static std::mutex mu;
    static int cache[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lk(mu);
    int& v = cache[dev & 63];
    if (v == 0) {
        cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
        if (v <= 0) v = 148;
    }
    return v;
}

}  // namespace kb

extern "C" const char* kb_status_str(int status) {
    switch (status) {
        case KB_OK: return "ok";
        case KB_ERR_INVALID_ARG: return "invalid argument (null pointer, negative size or bad flag)";
        case KB_ERR_UNSUPPORTED: return "unsupported shape, dtype, K or E";
        case KB_ERR_ALIGNMENT: return "pointer or stride not aligned as the kernel requires";
        case KB_ERR_WORKSPACE: return "workspace missing or smaller than the *_workspace_bytes size";
        case KB_ERR_TOO_LARGE: return "size overflows the int32 index space";
        case KB_ERR_SCRATCH_LIMIT:
            return "request exceeds the static scratch of kb_expert_maps_noalloc "
                   "(T <= 524288 tokens, workspace <= 8 MiB)";
        default: break;
    }
    if (status > 0) return cudaGetErrorString(static_cast<cudaError_t>(status));
    return "unknown status";
}

extern "C" int kb_version(void) { return 10000; }  // 1.0.0

extern "C" int kb_set_pdl(int enable) {
    return kb::g_pdl.exchange(enable ? 1 : 0);
}
