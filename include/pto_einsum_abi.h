/*
 * pto_einsum_abi.h - the extern "C" surface of one generated, cached einsum
 * library (build/<md5>/einsum_<md5>.so), i.e. the drop-in boundary the
 * reference's ctypes loader binds (builder.py:761-815).
 *
 * Every generated library is specialised to one equation, shapes and dtype;
 * `T` below is `float` for fp32 plans and `half` (fp16 bits carried as
 * uint16_t, ctypes.c_uint16) for fp16 plans. The output is always fp32.
 * Pointers are CUDA device pointers; `stream` is a cudaStream_t
 * (torch.cuda.current_stream().cuda_stream). The CUDA shims forward to the
 * core library declared in pto_einsum_b200.h.
 *
 * Symbol set per route (same as the reference templates):
 *   matmul route       all of the functions below
 *   elementwise route  run_einsum, run_einsum_setup/exec/exec_rc/teardown, run_einsum_last_error
 *   broadcast route    run_einsum, run_einsum_setup/exec/exec_rc/teardown, run_einsum_last_error
 */
#ifndef PTO_EINSUM_ABI_H
#define PTO_EINSUM_ABI_H

#include <stdint.h>

#ifndef PTO_EINSUM_HALF_DEFINED
#define PTO_EINSUM_HALF_DEFINED
typedef uint16_t half;  /* fp16 storage type across the C ABI */
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* One-shot contraction: setup + exec + stream synchronise + teardown.
 * Replaces templates.py:178-180 (run_einsum -> pto_einsum::einsum,
 * include/pto_einsum.h:283-290). */
void run_einsum(const void* input0, const void* input1, float* output, void* stream);

/* Allocate the persistent workspace for this plan; never returns NULL.
 * Replaces templates.py:181-183 (einsum_setup, include/pto_einsum.h:207-248). */
void* run_einsum_setup(void* stream);

/* Enqueue one contraction on `stream` (asynchronous).
 * Replaces templates.py:184-186 (einsum_exec, include/pto_einsum.h:253-275). */
void run_einsum_exec(const void* input0, const void* input1, float* output, void* workspace,
                     void* stream);

/* run_einsum_exec returning the call's status (0 or a pe_status code) instead
 * of void, so a caller needs one foreign call per contraction (new symbol, no
 * reference counterpart; run_einsum_exec forwards to it). */
int run_einsum_exec_rc(const void* input0, const void* input1, float* output, void* workspace,
                       void* stream);

/* Free the workspace. Replaces templates.py:187-189 (einsum_teardown,
 * include/pto_einsum.h:277-279). */
void run_einsum_teardown(void* workspace);

/* Standalone permutes of input0 / input1 into the canonical matmul layouts
 * ([I, L0, C] and [I, C, L1]) and of the [I, L0, L1] result into the output
 * order. Replace templates.py:166-174 (pto_einsum_transpose.h:662-678). */
void run_transpose_inp0(const void* input, void* output, void* stream);
void run_transpose_inp1(const void* input, void* output, void* stream);
void run_transpose_out(const float* input, float* output, void* stream);

/* Standalone batched matmul ws_res[I,L0,L1] = ws0[I,L0,C] x ws1[I,C,L1].
 * Replaces templates.py:175-177 (pto_einsum_matmul.h:973-1027). */
void run_batched_matmul(const void* ws0, const void* ws1, float* ws_res, void* stream);

/* New symbol (no reference counterpart): status of the last call made by this
 * host thread, 0 on success, a pe_status code otherwise. The reference entry
 * points return void and report nothing. */
int run_einsum_last_error(void);

#ifdef __cplusplus
}
#endif

#endif /* PTO_EINSUM_ABI_H */
