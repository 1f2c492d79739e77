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
std::atomic<long long> g_wait_limit{0};
}  // namespace

long long wait_limit(long long dflt) {
    const long long v = g_wait_limit.load(std::memory_order_relaxed);
    return v > 0 ? v : dflt;
}

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

extern "C" long long kb_set_wait_limit(long long polls) {
    return kb::g_wait_limit.exchange(polls > 0 ? polls : 0);
}

extern "C" int kb_workspace_status(const void* workspace, int kind, int* status,
                                   kb_stream_t stream) {
    if (!status) return KB_ERR_INVALID_ARG;
    const unsigned char* word = nullptr;
    if (kind == KB_WS_NOALLOC) {
        void* p = nullptr;
        const int st = kb::noalloc_scratch_address(&p);
        if (st) return st;
        word = static_cast<const unsigned char*>(p) + kb::maps_err_offset();
    } else if (kind == KB_WS_MAPS || kind == KB_WS_CHAIN || kind == KB_WS_EP ||
               kind == KB_WS_RGEMM) {
        if (!workspace) return KB_ERR_INVALID_ARG;
        word = static_cast<const unsigned char*>(workspace) +
               (kind == KB_WS_MAPS    ? kb::maps_err_offset()
                : kind == KB_WS_CHAIN ? kb::chain_err_offset()
                : kind == KB_WS_EP    ? kb::ep_err_offset()
                                      : 0);   // kb_router_gemm: the first word
    } else {
        return KB_ERR_INVALID_ARG;
    }
    int v = 0;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaMemcpyAsync(&v, word, sizeof(int), cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return static_cast<int>(e);
    *status = v;
    return KB_OK;
}
