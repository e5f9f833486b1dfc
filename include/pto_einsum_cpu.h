/*
 * pto_einsum_cpu.h - host (CPU) execution of a planned einsum, included by the
 * per-equation libraries EinsumBuilder generates for device="cpu".
 *
 * Same plan and same arithmetic as the reference's CPU path
 * (include/cpu_einsum.h:35-92 of vloncar/pto-einsum): every operand is
 * converted to fp32, each output element is accumulated in fp32 starting from
 * zero by adding the products over the contraction index c = 0, 1, ..., C-1
 * in that order, each product and each sum rounded once (no fused
 * multiply-add: build with -ffp-contract=off). So results are bit-identical to
 * the reference CPU path. The loop structure is this library's own:
 *  - operands are gathered once into the canonical [I, L0, C] / [I, C, L1]
 *    layouts (the reference's Phase A transposes) with 64-bit indices;
 *  - the product runs over groups of four output rows and blocks of 256 output
 *    columns with the four accumulator rows kept in cache and the c loop
 *    outermost inside the block, so the inner loop is a unit-stride vector
 *    update acc_r[j] += a_r * b[c][j] sharing each load of b between the four
 *    rows (per element still the reference's order);
 *  - rows of output are shared among host threads (std::thread); each element
 *    is computed by exactly one thread, so the thread count never changes a
 *    bit;
 *  - the result is written through the output permutation (Phase C).
 * The Hadamard route is out[i] = float(in0[i]) * float(in1[i]).
 * float16 inputs are rejected by the Python builder before this code is
 * generated, like the reference (builder.py:611-613).
 */
#ifndef PTO_EINSUM_CPU_H
#define PTO_EINSUM_CPU_H

#include <stdint.h>

#include <algorithm>
#include <thread>
#include <vector>

namespace pe_cpu {

/* Destination-order walk of a permute config (dims, to_shape, perm_strides):
 * calls f(dst_index, src_index) for every element. */
template <class P, class F>
inline void for_each_perm(F f) {
    constexpr unsigned D = P::dims;
    const int64_t n = (int64_t)P::N;
    if (n == 0) return;
    int64_t idx[D > 0 ? D : 1] = {0};
    int64_t src = 0;
    const int64_t inner = D ? P::to_shape[D - 1] : 1;
    const int64_t inner_st = D ? P::perm_strides[D - 1] : 0;
    for (int64_t base = 0; base < n; base += inner) {
        for (int64_t j = 0; j < inner; ++j) f(base + j, src + j * inner_st);
        // advance the outer odometer (axes D-2 .. 0)
        for (int a = (int)D - 2; a >= 0; --a) {
            src += P::perm_strides[a];
            if (++idx[a] < P::to_shape[a]) break;
            src -= P::perm_strides[a] * P::to_shape[a];
            idx[a] = 0;
        }
    }
}

/* Block updates of the product, compiled for AVX-512, AVX2 and baseline x86-64
 * and picked at load time (GNU ifunc). Vector lanes run over output columns
 * only, so each element still adds its products in c order, one rounding per
 * product and per sum (-ffp-contract=off keeps multiply and add separate). */
#if defined(__x86_64__) && defined(__GNUC__) && !defined(__clang__)
#define PE_CPU_CLONES __attribute__((target_clones("avx512f", "avx2", "default")))
#else
#define PE_CPU_CLONES
#endif

/* Four output rows o0..o3 (columns [0, nj)) = sum over c of a_r[c] * brow_c. */
PE_CPU_CLONES __attribute__((noinline)) static void block4(const float* a0p, int64_t C, const float* bcol,
                                                           int64_t L1, int64_t nj, float* __restrict o0,
                                                           float* __restrict o1, float* __restrict o2,
                                                           float* __restrict o3) {
    for (int64_t j = 0; j < nj; ++j) o0[j] = o1[j] = o2[j] = o3[j] = 0.0f;
    for (int64_t c = 0; c < C; ++c) {
        const float* __restrict brow = bcol + c * L1;
        const float a0 = a0p[c], a1 = a0p[C + c], a2 = a0p[2 * C + c], a3 = a0p[3 * C + c];
        for (int64_t j = 0; j < nj; ++j) {
            const float bv = brow[j];
            o0[j] = o0[j] + a0 * bv;
            o1[j] = o1[j] + a1 * bv;
            o2[j] = o2[j] + a2 * bv;
            o3[j] = o3[j] + a3 * bv;
        }
    }
}

/* One output row. */
PE_CPU_CLONES __attribute__((noinline)) static void block1(const float* arow, int64_t C, const float* bcol,
                                                           int64_t L1, int64_t nj, float* __restrict o0) {
    for (int64_t j = 0; j < nj; ++j) o0[j] = 0.0f;
    for (int64_t c = 0; c < C; ++c) {
        const float* __restrict brow = bcol + c * L1;
        const float a0 = arow[c];
        for (int64_t j = 0; j < nj; ++j) o0[j] = o0[j] + a0 * brow[j];
    }
}

template <class F>
inline void parallel_rows(int64_t rows, int64_t work_per_row, F f) {
    unsigned hw = std::thread::hardware_concurrency();
    int64_t nt = hw ? hw : 1;
    // about 1M multiply-adds per thread at least, so small problems stay serial
    nt = std::min<int64_t>(nt, std::max<int64_t>(1, rows * work_per_row / (int64_t)(1 << 20)));
    nt = std::min<int64_t>(nt, rows);
    if (nt <= 1) {
        f(0, rows);
        return;
    }
    std::vector<std::thread> th;
    const int64_t per = (rows + nt - 1) / nt;
    int64_t t = 0;
    for (; t < nt; ++t) {
        const int64_t lo = t * per, hi = std::min(rows, lo + per);
        if (lo >= hi) break;
        try {
            th.emplace_back([=, &f] { f(lo, hi); });
        } catch (...) {
            break;  // no thread could be started (resource limits): finish here
        }
    }
    if (t * per < rows) f(t * per, rows);
    for (auto& x : th) x.join();
}

/* res = permute_out(batched_matmul(permute_in0(data0), permute_in1(data1))). */
template <typename T, class E>
inline int einsum(const T* data0, const T* data1, float* res) {
    typedef typename E::tpose_inp0_config P0;
    typedef typename E::tpose_inp1_config P1;
    typedef typename E::tpose_out_conf PO;
    const int64_t I = E::n_inplace, L0 = E::n_free0, L1 = E::n_free1, C = E::n_contract;
    std::vector<float> a, b, o;
    try {
        a.resize((size_t)P0::N);
        b.resize((size_t)P1::N);
        o.resize((size_t)PO::N);
    } catch (...) {
        return 1;  // host memory exhausted: reported, nothing written
    }
    for_each_perm<P0>([&](int64_t d, int64_t s) { a[(size_t)d] = static_cast<float>(data0[s]); });
    for_each_perm<P1>([&](int64_t d, int64_t s) { b[(size_t)d] = static_cast<float>(data1[s]); });
    constexpr int64_t JB = 256;  // output columns per block (1 KB accumulator row)
    constexpr int64_t RB = 4;    // output rows sharing each loaded row of B
    const float* A = a.data();
    const float* B = b.data();
    float* O = o.data();
    // work items: (batch, group of RB rows); rows of a group share their B loads
    const int64_t groups = (L0 + RB - 1) / RB;
    parallel_rows(I * groups, RB * L1 * C, [&](int64_t g0, int64_t g1) {
        for (int64_t g = g0; g < g1; ++g) {
            const int64_t i = g / groups;
            const int64_t l0 = (g - i * groups) * RB;
            const int64_t nr = std::min(RB, L0 - l0);
            const float* bmat = B + i * C * L1;
            for (int64_t j0 = 0; j0 < L1; j0 += JB) {
                const int64_t nj = std::min(JB, L1 - j0);
                if (nr == RB) {
                    float* o0 = O + (i * L0 + l0) * L1 + j0;
                    block4(A + (i * L0 + l0) * C, C, bmat + j0, L1, nj, o0, o0 + L1, o0 + 2 * L1, o0 + 3 * L1);
                } else {
                    for (int64_t r = 0; r < nr; ++r)
                        block1(A + (i * L0 + l0 + r) * C, C, bmat + j0, L1, nj, O + (i * L0 + l0 + r) * L1 + j0);
                }
            }
        }
    });
    for_each_perm<PO>([&](int64_t d, int64_t s) { res[d] = O[s]; });
    return 0;
}

/* Hadamard product. */
template <typename T, class E>
inline int elementwise_mul(const T* in0, const T* in1, float* res) {
    const int64_t n = (int64_t)E::N;
    parallel_rows(n, 1, [&](int64_t lo, int64_t hi) {
        for (int64_t k = lo; k < hi; ++k) res[k] = static_cast<float>(in0[k]) * static_cast<float>(in1[k]);
    });
    return 0;
}

}  // namespace pe_cpu

#endif /* PTO_EINSUM_CPU_H */
