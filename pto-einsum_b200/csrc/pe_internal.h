// pe_internal.h - declarations shared between the core library's translation units.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "pto_einsum_b200.h"

namespace pe {

int set_last_error(int code);
int check_cuda(cudaError_t e);
int num_sms();
void count_launch(int n = 1);

int elementwise_mul(int32_t dtype, const void* a, const void* b, float* out, int64_t n,
                    cudaStream_t s);
int broadcast_mul(const pe_broadcast_plan* pl, const void* full, const void* bc, float* out,
                  cudaStream_t s);
int permute(const pe_permute_plan* pl, const void* in, void* out, cudaStream_t s);

// Generic strided copy over a logical index space (outermost axis first).
int strided_copy_launch(int es, int nd, const int64_t* size, const int64_t* sst,
                        const int64_t* dst_st, const void* src, void* dst, cudaStream_t s);

int contract_workspace_bytes(const pe_contract_plan* plan, size_t* bytes);
// Scratch bytes pe_contract needs for these exact input pointers.
int contract_scratch_bytes(const pe_contract_plan* plan, const void* in0, const void* in1, size_t* bytes);
int contract(const pe_contract_plan* plan, const void* in0, const void* in1, float* out, void* ws,
             size_t ws_bytes, cudaStream_t s);

// Prepared-launch cache held by a workspace handle: contract_cached replays the
// launches of an earlier call with the same plan object and pointers.
void* program_cache_create();
void program_cache_destroy(void* cache);
// phase: EINSUM_PHASE_STOP level (3 = the full contraction)
int contract_cached(void* cache, const pe_contract_plan* plan, const void* in0, const void* in1, float* out,
                    void* ws, size_t ws_bytes, int phase, cudaStream_t s);

// Read (and optionally clear) the device error word of the GEMM kernels.
int gemm_device_error(bool clear);
int wait_timeout_selftest(uint64_t timeout_ns, cudaStream_t s);

}  // namespace pe
