/*
 * pto_einsum_b200.h - C ABI of the prebuilt sm_100a einsum core library
 * (libpto_einsum_b200.so).
 *
 * The per-equation shared objects that EinsumBuilder generates and caches
 * (build/<md5>/einsum_<md5>.so, see pto_einsum_abi.h) are thin C++ shims:
 * they hold the plan as constexpr config structs and forward every call to
 * the functions below. All device work (permutes, tcgen05 GEMM, streaming
 * multiplies) lives in this one library, compiled once for sm_100a.
 *
 * Conventions
 *  - Every pointer is a device pointer unless stated otherwise. Inputs are
 *    C-contiguous, the output is fp32 C-contiguous in the planned order.
 *  - `stream` is a cudaStream_t passed as void* (torch.cuda.current_stream()
 *    .cuda_stream). All calls only enqueue work on that stream.
 *  - Functions return 0 on success or a PE_ERR_* code; the code is also
 *    remembered per thread and readable through pe_last_error().
 *  - Device-side faults that the kernels detect themselves (a pipeline wait
 *    that ran out of time) are recorded in a device word read with
 *    pe_device_error(), which synchronises the stream.
 */
#ifndef PTO_EINSUM_B200_H
#define PTO_EINSUM_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PE_MAX_RANK 8

enum pe_dtype { PE_F32 = 0, PE_F16 = 1 };

enum pe_status {
    PE_OK = 0,
    PE_ERR_INVALID = 1,      /* bad plan / argument */
    PE_ERR_UNSUPPORTED = 2,  /* plan outside what the backend lowers */
    PE_ERR_CUDA = 3,         /* a CUDA runtime call failed */
    PE_ERR_NO_DEVICE = 4,    /* no sm_100 device / driver entry point */
    PE_ERR_WORKSPACE = 5,    /* workspace missing or too small */
    PE_ERR_TIMEOUT = 6,      /* a kernel pipeline wait gave up (device word) */
    PE_ERR_DEVICE = 7        /* other device-detected fault (device word) */
};

/*
 * Two-operand contraction plan: transpose -> batched matmul -> transpose.
 * Mirrors the reference recipe (builder.py:44-110, templates.py:1-62):
 *   perm0 = in_transpose_idxs[0] = batch axes + free0 axes + contract axes
 *   perm1 = in_transpose_idxs[1] = batch axes + contract axes + free1 axes
 *   out_interp_shape = batch + free0 + free1 sizes, out_perm = out_transpose_idxs
 * n_batch/n_free0/n_free1/n_contract are the axis counts of each group.
 */
typedef struct pe_contract_plan {
    int32_t dtype;                       /* pe_dtype of both inputs */
    int32_t rank0, rank1, out_rank;
    int64_t shape0[PE_MAX_RANK];
    int64_t shape1[PE_MAX_RANK];
    int32_t perm0[PE_MAX_RANK];
    int32_t perm1[PE_MAX_RANK];
    int64_t out_interp_shape[PE_MAX_RANK];
    int32_t out_perm[PE_MAX_RANK];
    int32_t n_batch, n_free0, n_free1, n_contract;
    int64_t I, L0, L1, C;
} pe_contract_plan;

/*
 * Broadcast multiply plan (builder.py:369-447, templates.py:94-105):
 * out[e] = full[e] * bc[boff(e)], boff(e) = sum_q idx_q(e / Inner) *
 * outer_bstride[q] + (mode == 0 ? e % Cc : 0).
 */
typedef struct pe_broadcast_plan {
    int32_t dtype;
    int32_t mode;                        /* 0 column-expand, 1 scalar per group */
    int64_t n, Cc, Rr, Inner, Outer, sizeB;
    int32_t outer_rank;
    int64_t outer_dims[PE_MAX_RANK];
    int64_t outer_bstride[PE_MAX_RANK];
} pe_broadcast_plan;

/* N-D permute (builder.py:449-461): out = in.permute(perm).contiguous(). */
typedef struct pe_permute_plan {
    int32_t dtype;                       /* element type of in and out */
    int32_t dims;
    int64_t from_shape[PE_MAX_RANK];
    int32_t perm[PE_MAX_RANK];
} pe_permute_plan;

/* ---- contraction ------------------------------------------------------ */

/* Device bytes of scratch that pe_contract needs for this plan (0 if none). */
int pe_contract_workspace_bytes(const pe_contract_plan* plan, size_t* bytes);

/* Enqueue the contraction. ws may be NULL only if the workspace size is 0. */
int pe_contract(const pe_contract_plan* plan, const void* in0, const void* in1,
                float* out, void* ws, size_t ws_bytes, void* stream);

/*
 * Persistent workspace handle (replaces the reference's einsum_setup /
 * einsum_teardown, include/pto_einsum.h:207-279). Never returns NULL: a plan
 * that needs no scratch gets a token handle. pe_workspace_ptr/bytes expose
 * the device buffer held by the handle.
 */
void* pe_workspace_create(const pe_contract_plan* plan, void* stream);
/*
 * pe_contract with the scratch held by `handle` (pe_workspace_create), the
 * per-call path of the generated run_einsum_exec (reference einsum_exec,
 * include/pto_einsum.h:253-275). The handle also remembers the prepared
 * launches (lowered plan, encoded tensor maps) of its last 8 distinct
 * (plan, in0, in1, out) combinations, so a repeated call only enqueues its
 * kernels. Calls on one handle are serialised by a lock.
 */
int pe_contract_ws(void* handle, const pe_contract_plan* plan, const void* in0, const void* in1,
                   float* out, void* stream);
/*
 * Phase-gated pe_contract_ws for profiling (the reference's EINSUM_PHASE_STOP
 * gate, include/pto_einsum.h:18-30, driven by
 * benchmarks/profile_phase_overlap.py:72-93): the fused kernel keeps its launch
 * and pipeline-barrier skeleton at every level and runs its work up to
 *   0 = barriers only, 1 = + operand loads (TMA, gather pre-pass, tf32 split),
 *   2 = + tensor-core MMAs, 3 = + epilogue stores and split-K reduction (full).
 * Below 3 the output is not written. Single-phase streaming contractions
 * (degenerate and thin shapes) launch nothing below 3. A generated library
 * built with EINSUM_EXTRA_DEFINES="-DEINSUM_PHASE_STOP=N" calls this from its
 * run_einsum_exec.
 */
int pe_contract_ws_phase(void* handle, const pe_contract_plan* plan, const void* in0, const void* in1,
                         float* out, int phase_stop, void* stream);
void* pe_workspace_ptr(void* handle);
size_t pe_workspace_size(void* handle);
void pe_workspace_destroy(void* handle);

/* Canonical batched matmul: c[I,L0,L1] = a[I,L0,C] x b[I,C,L1] (fp32 out). */
int pe_batched_matmul(int32_t dtype, int64_t I, int64_t L0, int64_t L1, int64_t C,
                      const void* a, const void* b, float* c, void* stream);

/*
 * Allocation-free contraction (no counterpart in the reference). Same result
 * as pe_contract, but the scratch it may need (gathered operands, split-K
 * partial sums) comes from a fixed 32 MiB array compiled into this library
 * instead of cudaMalloc, for callers that cannot allocate device memory at
 * call time (fixed memory budgets, foreign allocators, latency-critical
 * paths). The array occupies 32 MiB on every GPU that uses the library until
 * the process exits.
 *  - Plans needing more scratch than pe_noalloc_scratch_bytes() are rejected
 *    with PE_ERR_WORKSPACE before anything is launched.
 *  - The first call on each device looks up the array's device address
 *    (cudaGetSymbolAddress) with that device current; make that first call
 *    before any stream capture. The address is cached per device for the life
 *    of the process; it is not valid after cudaDeviceReset (or after the
 *    primary context is released and created again), so do not call this
 *    entry point after resetting a device.
 *  - All calls share the one array: calls whose kernels can overlap on the GPU
 *    (different streams, or several host threads) race on it and must be
 *    serialised by the caller. Nothing in it needs to start zeroed; every
 *    byte a call reads was written earlier by the same call.
 */
int pe_contract_noalloc(const pe_contract_plan* plan, const void* in0, const void* in1,
                        float* out, void* stream);
/* Size in bytes of the fixed scratch array behind pe_contract_noalloc. */
size_t pe_noalloc_scratch_bytes(void);

/* ---- streaming multiplies ------------------------------------------------ */

/* Hadamard product out[i] = float(a[i]) * float(b[i]), i < n. */
int pe_elementwise_mul(int32_t dtype, const void* a, const void* b, float* out,
                       int64_t n, void* stream);

/* Broadcast multiply (see pe_broadcast_plan). */
int pe_broadcast_mul(const pe_broadcast_plan* plan, const void* full, const void* bc,
                     float* out, void* stream);

/* ---- permute --------------------------------------------------------------- */

int pe_permute(const pe_permute_plan* plan, const void* in, void* out, void* stream);

/* ---- status ---------------------------------------------------------------- */

/* Status of the last pe_* call made by this host thread. */
int pe_last_error(void);
/* Human readable text of a status code. */
const char* pe_error_string(int code);
/* Synchronise `stream`, return and clear the device-side error word. */
int pe_device_error(void* stream);
/* Self-test of the device-side failure path: one CTA waits on a pipeline barrier
 * that nothing arrives on, through the same bounded wait every GEMM stage uses,
 * with a limit of `timeout_ns` (at most 100 ms). Returns the device error word the
 * expired wait recorded (PE_ERR_TIMEOUT | site << 8, site 15) and clears it; the
 * CUDA context stays usable. Synchronises `stream`. */
int pe_selftest_wait_timeout(uint64_t timeout_ns, void* stream);
/* Number of core kernels this process has launched (for launch accounting). */
int64_t pe_launch_count(void);
/* Block the host until all work queued on `stream` finished. */
int pe_stream_synchronize(void* stream);
/* Library build tag, e.g. "pto_einsum_b200 sm_100a <hash>". */
const char* pe_version(void);

#ifdef __cplusplus
}
#endif

#endif /* PTO_EINSUM_B200_H */
