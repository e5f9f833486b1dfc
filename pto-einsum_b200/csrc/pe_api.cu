// pe_api.cu - extern "C" entry points of libpto_einsum_b200.so, status and
// workspace handling.
//
// The workspace handle replaces the reference's einsum_setup / einsum_exec /
// einsum_teardown trio (include/pto_einsum.h:207-279): setup sizes and
// allocates the scratch the plan needs once, exec only enqueues kernels.
#include <atomic>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "pe_common.cuh"

#ifndef PE_BUILD_TAG
#define PE_BUILD_TAG "dev"
#endif

namespace pe {

namespace {
thread_local int t_last_error = PE_OK;
std::atomic<int64_t> g_launches{0};

struct Workspace {
    uint32_t magic;
    void* ptr;
    size_t bytes;
    int device;
    void* cache;   // prepared launches of recent calls (pe_contract_ws)
};
constexpr uint32_t kMagic = 0x50455753u;  // "PEWS"
}  // namespace

int set_last_error(int code) {
    t_last_error = code;
    return code;
}

int check_cuda(cudaError_t e) {
    if (e == cudaSuccess) return set_last_error(PE_OK);
    return set_last_error(PE_ERR_CUDA);
}

int num_sms() {
    // cached per device (the reference caches its core count the same way,
    // pto_einsum_utils.h:124-133)
    static int cache[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    if (cache[dev] == 0) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
            n = 148;
        cache[dev] = n;
    }
    return cache[dev];
}

void count_launch(int n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

}  // namespace pe

using namespace pe;

extern "C" {

int pe_contract_workspace_bytes(const pe_contract_plan* plan, size_t* bytes) {
    return contract_workspace_bytes(plan, bytes);
}

int pe_contract(const pe_contract_plan* plan, const void* in0, const void* in1, float* out, void* ws,
                size_t ws_bytes, void* stream) {
    return contract(plan, in0, in1, out, ws, ws_bytes, (cudaStream_t)stream);
}

int pe_contract_ws(void* handle, const pe_contract_plan* plan, const void* in0, const void* in1, float* out,
                   void* stream) {
    Workspace* w = (Workspace*)handle;
    if (!w || w->magic != kMagic) return set_last_error(PE_ERR_WORKSPACE);
    return contract_cached(w->cache, plan, in0, in1, out, w->ptr, w->bytes, 3, (cudaStream_t)stream);
}

int pe_contract_ws_phase(void* handle, const pe_contract_plan* plan, const void* in0, const void* in1,
                         float* out, int phase_stop, void* stream) {
    Workspace* w = (Workspace*)handle;
    if (!w || w->magic != kMagic) return set_last_error(PE_ERR_WORKSPACE);
    if (phase_stop < 0 || phase_stop > 3) return set_last_error(PE_ERR_INVALID);
    return contract_cached(w->cache, plan, in0, in1, out, w->ptr, w->bytes, phase_stop, (cudaStream_t)stream);
}

void* pe_workspace_create(const pe_contract_plan* plan, void* stream) {
    Workspace* w = new Workspace{kMagic, nullptr, 0, 0, program_cache_create()};
    cudaGetDevice(&w->device);
    size_t bytes = 0;
    if (plan && contract_workspace_bytes(plan, &bytes) == PE_OK && bytes > 0) {
        if (cudaMalloc(&w->ptr, bytes) == cudaSuccess) {
            w->bytes = bytes;
            set_last_error(PE_OK);
        } else {
            // not sticky: clear the runtime's last-error slot so later launch
            // checks on this thread do not report this failure again
            (void)cudaGetLastError();
            w->ptr = nullptr;
            set_last_error(PE_ERR_CUDA);
        }
    }
    (void)stream;
    return w;
}

void* pe_workspace_ptr(void* handle) {
    Workspace* w = (Workspace*)handle;
    return (w && w->magic == kMagic) ? w->ptr : nullptr;
}

size_t pe_workspace_size(void* handle) {
    Workspace* w = (Workspace*)handle;
    return (w && w->magic == kMagic) ? w->bytes : 0;
}

void pe_workspace_destroy(void* handle) {
    Workspace* w = (Workspace*)handle;
    if (!w || w->magic != kMagic) return;
    if (w->ptr) cudaFree(w->ptr);
    program_cache_destroy(w->cache);
    w->magic = 0;
    delete w;
}

int pe_batched_matmul(int32_t dtype, int64_t I, int64_t L0, int64_t L1, int64_t C, const void* a,
                      const void* b, float* c, void* stream) {
    pe_contract_plan p;
    memset(&p, 0, sizeof(p));
    p.dtype = dtype;
    p.rank0 = p.rank1 = p.out_rank = 3;
    p.shape0[0] = I; p.shape0[1] = L0; p.shape0[2] = C;
    p.shape1[0] = I; p.shape1[1] = C; p.shape1[2] = L1;
    for (int j = 0; j < 3; ++j) { p.perm0[j] = j; p.perm1[j] = j; p.out_perm[j] = j; }
    p.out_interp_shape[0] = I; p.out_interp_shape[1] = L0; p.out_interp_shape[2] = L1;
    p.n_batch = p.n_free0 = p.n_free1 = p.n_contract = 1;
    p.I = I; p.L0 = L0; p.L1 = L1; p.C = C;
    return contract(&p, a, b, c, nullptr, 0, (cudaStream_t)stream);
}

int pe_elementwise_mul(int32_t dtype, const void* a, const void* b, float* out, int64_t n,
                       void* stream) {
    return elementwise_mul(dtype, a, b, out, n, (cudaStream_t)stream);
}

int pe_broadcast_mul(const pe_broadcast_plan* plan, const void* full, const void* bc, float* out,
                     void* stream) {
    return broadcast_mul(plan, full, bc, out, (cudaStream_t)stream);
}

int pe_permute(const pe_permute_plan* plan, const void* in, void* out, void* stream) {
    return permute(plan, in, out, (cudaStream_t)stream);
}

int pe_last_error(void) { return t_last_error; }

const char* pe_error_string(int code) {
    switch (code & 0xFF) {
        case PE_OK: return "ok";
        case PE_ERR_INVALID: return "invalid plan or argument";
        case PE_ERR_UNSUPPORTED: return "plan not supported by the CUDA backend";
        case PE_ERR_CUDA: return "CUDA runtime error";
        case PE_ERR_NO_DEVICE: return "no usable sm_100 device or driver entry point";
        case PE_ERR_WORKSPACE: return "workspace missing or too small";
        case PE_ERR_TIMEOUT: return "device pipeline wait timed out";
        case PE_ERR_DEVICE: return "device-detected fault";
        default: return "unknown error";
    }
}

int pe_device_error(void* stream) {
    if (cudaStreamSynchronize((cudaStream_t)stream) != cudaSuccess) return set_last_error(PE_ERR_CUDA);
    int v = gemm_device_error(true);
    if (v < 0) return set_last_error(PE_ERR_CUDA);
    set_last_error(PE_OK);
    return v;
}

int pe_selftest_wait_timeout(uint64_t timeout_ns, void* stream) {
    return wait_timeout_selftest(timeout_ns, (cudaStream_t)stream);
}

int pe_stream_synchronize(void* stream) {
    return check_cuda(cudaStreamSynchronize((cudaStream_t)stream));
}

int64_t pe_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

const char* pe_version(void) { return "pto_einsum_b200 sm_100a " PE_BUILD_TAG; }

}  // extern "C"
