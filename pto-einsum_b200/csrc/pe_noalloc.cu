// pe_noalloc.cu - a contraction entry point that allocates no device memory.
//
// pe_contract() needs scratch for two things: operands that a TMA tensor map
// cannot read in place (gathered into a canonical layout) and split-K partial
// sums. Normally that scratch comes from pe_workspace_create(), i.e. from
// cudaMalloc. Some callers cannot allocate at call time: code running under a
// fixed memory budget or a custom allocator that must not see foreign
// allocations, plugins loaded into a host whose device memory is owned
// elsewhere, and latency-critical paths where a cudaMalloc (which can
// synchronise the device) is not acceptable. pe_contract_noalloc() serves
// them: its scratch is a fixed array compiled into this library.
//
// The array below lives in device memory on every GPU where the library is
// loaded, from the first use until the process exits. Host code must not
// pass the symbol itself to a kernel (on the host it is only a stand-in, not
// a device address); the device address is looked up once per device with
// cudaGetSymbolAddress while that device is current.
#include <mutex>

#include "pe_common.cuh"

namespace pe {

namespace {

constexpr size_t kNoAllocScratchBytes = 32u << 20;  // 32 MiB per device

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_mu;
void* g_scratch_ptr[64] = {nullptr};

// Device address of the scratch array on the current device (looked up once).
int scratch_address(void** out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return set_last_error(PE_ERR_CUDA);
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_scratch_ptr[dev]) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p) return set_last_error(PE_ERR_CUDA);
        g_scratch_ptr[dev] = p;
    }
    *out = g_scratch_ptr[dev];
    return PE_OK;
}

}  // namespace

}  // namespace pe

using namespace pe;

extern "C" {

size_t pe_noalloc_scratch_bytes(void) { return kNoAllocScratchBytes; }

int pe_contract_noalloc(const pe_contract_plan* plan, const void* in0, const void* in1, float* out,
                        void* stream) {
    // Exact scratch need for these pointers (alignment decides which operands
    // are read in place), then the existing contraction with the fixed array
    // as its workspace. Because the array is at least as large as the need,
    // pe_contract never falls back to its own stream-ordered allocation.
    size_t need = 0;
    int rc = contract_scratch_bytes(plan, in0, in1, &need);
    if (rc) return rc;
    if (need > kNoAllocScratchBytes) return set_last_error(PE_ERR_WORKSPACE);
    void* scratch = nullptr;
    if (need > 0) {
        rc = scratch_address(&scratch);
        if (rc) return rc;
    }
    return contract(plan, in0, in1, out, scratch, need > 0 ? kNoAllocScratchBytes : 0, (cudaStream_t)stream);
}

}  // extern "C"
