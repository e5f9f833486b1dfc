/*
 * einsum_oracle.c - TEST INFRASTRUCTURE ONLY (parity checker, CPU baseline).
 *
 * Plain-C restatement of the reference CPU path, include/cpu_einsum.h:
 *   transfer_idx / transpose   cpu_einsum.h:35-51  (div/mod index decode)
 *   einsum                     cpu_einsum.h:53-83  (transpose both inputs,
 *                               I x L0 x L1 x C loop, fp32 accumulate in
 *                               increasing c, transpose the result)
 *   elementwise_mul            cpu_einsum.h:87-92
 * plus the broadcast multiply that the reference NPU path computes
 * (pto_einsum_elementwise.h:129-370; one exact product per element).
 *
 * Shapes are runtime arguments instead of constexpr config structs. The
 * matmul may split rows across threads; each output element is still
 * accumulated by one thread in the reference order, so results do not depend
 * on the thread count. Build with -ffp-contract=off so a*b+acc is never fused
 * (the reference's x86-64 g++ -O3 build has no FMA either).
 */
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* cpu_einsum.h:35-43: flat output index -> flat input index */
static int64_t transfer_idx(int64_t index, int dims, const int64_t* to_shape, const int64_t* perm_strides) {
    int64_t idx = 0;
    for (int i = dims - 1; i >= 0; i--) {
        idx += (index % to_shape[i]) * perm_strides[i];
        index /= to_shape[i];
    }
    return idx;
}

/* cpu_einsum.h:45-51 */
int oracle_transpose_f32(const float* data, float* res, int dims, const int64_t* to_shape,
                         const int64_t* perm_strides) {
    int64_t n = 1;
    for (int i = 0; i < dims; i++) n *= to_shape[i];
    for (int64_t i = 0; i < n; i++) res[i] = data[transfer_idx(i, dims, to_shape, perm_strides)];
    return 0;
}

typedef struct {
    const float *a, *b;
    float* o;
    int64_t I, L0, L1, C;
    int64_t row_begin, row_end; /* rows of the flattened [I*L0] range */
} mm_task;

/* cpu_einsum.h:67-80, for rows [row_begin, row_end) of the [I*L0] range */
static void* mm_worker(void* arg) {
    mm_task* t = (mm_task*)arg;
    const int64_t L0 = t->L0, L1 = t->L1, C = t->C;
    for (int64_t row = t->row_begin; row < t->row_end; row++) {
        const int64_t i = row / L0;
        const float* arow = t->a + row * C;
        const float* bmat = t->b + i * L1 * C;
        float* orow = t->o + row * L1;
        for (int64_t l1 = 0; l1 < L1; l1++) {
            float acc = 0.0f;
            for (int64_t c = 0; c < C; c++) acc += arow[c] * bmat[c * L1 + l1];
            orow[l1] = acc;
        }
    }
    return NULL;
}

/* Canonical batched matmul o[I,L0,L1] = a[I,L0,C] x b[I,C,L1]. */
int oracle_batched_matmul_f32(const float* a, const float* b, float* o, int64_t I, int64_t L0, int64_t L1,
                              int64_t C, int nthreads) {
    int64_t rows = I * L0;
    if (nthreads < 1) nthreads = 1;
    if (nthreads > 256) nthreads = 256;
    if (rows < nthreads) nthreads = rows > 0 ? (int)rows : 1;
    mm_task tasks[256];
    pthread_t th[256];
    for (int t = 0; t < nthreads; t++) {
        tasks[t] = (mm_task){a, b, o, I, L0, L1, C, rows * t / nthreads, rows * (t + 1) / nthreads};
    }
    if (nthreads == 1) {
        mm_worker(&tasks[0]);
        return 0;
    }
    for (int t = 0; t < nthreads; t++) pthread_create(&th[t], NULL, mm_worker, &tasks[t]);
    for (int t = 0; t < nthreads; t++) pthread_join(th[t], NULL);
    return 0;
}

/* cpu_einsum.h:53-83 with runtime shapes. */
int oracle_einsum_f32(const float* in0, const float* in1, float* out, int d0, const int64_t* to0,
                      const int64_t* ps0, int d1, const int64_t* to1, const int64_t* ps1, int dout,
                      const int64_t* too, const int64_t* pso, int64_t I, int64_t L0, int64_t L1, int64_t C,
                      int nthreads) {
    float* t0 = (float*)malloc(sizeof(float) * (size_t)(I * L0 * C > 0 ? I * L0 * C : 1));
    float* t1 = (float*)malloc(sizeof(float) * (size_t)(I * C * L1 > 0 ? I * C * L1 : 1));
    float* to = (float*)malloc(sizeof(float) * (size_t)(I * L0 * L1 > 0 ? I * L0 * L1 : 1));
    if (!t0 || !t1 || !to) {
        free(t0);
        free(t1);
        free(to);
        return 1;
    }
    oracle_transpose_f32(in0, t0, d0, to0, ps0);
    oracle_transpose_f32(in1, t1, d1, to1, ps1);
    oracle_batched_matmul_f32(t0, t1, to, I, L0, L1, C, nthreads);
    oracle_transpose_f32(to, out, dout, too, pso);
    free(t0);
    free(t1);
    free(to);
    return 0;
}

/* cpu_einsum.h:87-92 */
int oracle_elementwise_f32(const float* a, const float* b, float* out, int64_t n) {
    for (int64_t i = 0; i < n; i++) out[i] = a[i] * b[i];
    return 0;
}

/* out[e] = full[e] * bc[boff(e)]: the broadcast route's definition
 * (builder.py:369-447, pto_einsum_elementwise.h:129-370). */
int oracle_broadcast_f32(const float* full, const float* bc, float* out, int mode, int64_t n, int64_t Cc,
                         int64_t Inner, int outer_rank, const int64_t* outer_dims, const int64_t* outer_bstride) {
    for (int64_t e = 0; e < n; e++) {
        int64_t o = e / Inner, boff = 0;
        for (int q = outer_rank - 1; q >= 0; q--) {
            boff += (o % outer_dims[q]) * outer_bstride[q];
            o /= outer_dims[q];
        }
        if (mode == 0) boff += (e % Inner) % Cc;
        out[e] = full[e] * bc[boff];
    }
    return 0;
}
