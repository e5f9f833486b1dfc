// pe_gemm.cu - fused contraction: strided TMA loads -> tcgen05/TMEM batched
// GEMM -> permuted epilogue store, one persistent launch per contraction.
//
// Replaces the Ascend mix kernel einsum_fused_kernel (include/pto_einsum.h:65-177)
// and its batched matmul schedules (include/pto_einsum_matmul.h:115-970):
//  * Phase A (input permute) becomes TMA addressing: each operand is described
//    by a rank-5 tensor map over the caller's tensor (free axis, contraction
//    axis, up to three batch axes, any strides), read K-major or MN-major.
//    Out-of-range rows/columns/contraction entries arrive as zeros, which is
//    the K-padding and boundary-tile handling of matmul.h:33-65 without a copy.
//    Operands a tensor map cannot describe are first gathered by pe_permute.cu
//    into a canonical [batch, free, K] workspace.
//  * Phase B is a warp-specialised persistent kernel: warp 0 issues TMA loads
//    into a STAGES-deep shared-memory ring, one thread of warp 1 issues
//    tcgen05.mma into a double-buffered TMEM accumulator, warps 2-5 drain the
//    other accumulator while the next tile is multiplied.
//  * Phase C (output permute) is fused into the epilogue: tcgen05.ld in the
//    16x256b layout -> full-sector 8-byte stores into the permuted output when
//    its rows are unit-stride (16-byte aligned strides), else strided stores
//    decoded per row and column.
//  fp16 operands use kind::f16 with fp32 accumulation. fp32 operands use
//  kind::tf32 in the 3xTF32 scheme: x = big + small with big = x with the low
//  13 mantissa bits cleared (exactly representable in tf32) and small = x - big;
//  D += As*Bb + Ab*Bs + Ab*Bb, which restores ~fp32 accuracy. Warps 6-9 do the
//  split in shared memory between the TMA landing and the MMA.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstring>
#include <functional>
#include <mutex>
#include <vector>

#include <cuda_fp16.h>

#include "pe_common.cuh"

namespace pe {

namespace {

constexpr int kMaxBatchMap = 3;

struct MapBatch {
    int nb;
    uint32_t size[kMaxBatchMap];
    uint32_t div[kMaxBatchMap];
};

struct Decode {
    int n;
    int64_t size[PE_MAX_RANK];
    int64_t stride[PE_MAX_RANK];
};

struct GemmArgs {
    CUtensorMap tma;
    CUtensorMap tmb;
    CUtensorMap tmas;   // fp32: precomputed tf32 "small" halves of A / B (same layout)
    CUtensorMap tmbs;
    int a_pre, b_pre;   // fp32: operand's small half comes from tmas / tmbs
    int M, N, K;
    int mblk, nblk, tiles, kiters;
    int a_mn, b_mn;
    MapBatch ab, bb;
    int out_rows;    // output rows unit-stride with 16-byte aligned strides (full-sector stores)
    int out_v8;      // and 32-byte aligned rows: full-line 32-byte stores after a quad transpose
    int acc_slots;   // fp32: accumulator slots per tile (1, 2 or 4)
    int fuse_b;      // fp32, 128-column single-CTA tiles: one N=256 MMA Ab x [Bb | Bs] and one
                     // N=128 MMA As x Bb per k-step; B's small half lands right after B, A's
                     // after it; two k-rotation slots of two 128-column halves (acc_slots = 4)
    int ksplit;      // work units per output tile (split-K), >= 1
    int kper;        // k-iterations per unit
    int sk_q;        // stream-K: k-iterations per CTA (group) over the flattened (tile, k) space; 0 = off
    int nbatch;      // I: batch count of the plan (split-K partials use batch i + sp*I)
    int raw_big;     // fp32: feed x unmasked as the big part (tensor core truncation)
    int phase;       // phases run (EINSUM_PHASE_STOP): 0 pipeline barriers only, 1 + operand
                     // loads, 2 + tensor-core MMAs, 3 + epilogue stores (the full kernel)
    float* out;
    Decode ob, om, on;
};

template <int BN_, bool F32_, int EPIW_ = (F32_ ? 4 : 8), bool PAIR_ = false, int SPLITW_ = (F32_ ? 4 : 0),
          int KB_ = 1>
struct Cfg {
    // PAIR: a cluster of two CTAs computes one TM = 256-row tile with
    // tcgen05 cta_group::2; each CTA lands 128 rows of A and half of B's N.
    static constexpr bool PAIR = PAIR_;
    static constexpr int BM = 128;                      // rows of A per CTA
    static constexpr int TM = PAIR ? 256 : 128;         // rows of the output tile
    static constexpr int BN = BN_;
    static constexpr bool F32 = F32_;
    static constexpr int ES = F32 ? 4 : 2;
    // KB 128-byte swizzle rows of the contraction per stage: K-major operands
    // land as KB boxes side by side (each a [rows][128 B] block), MN-major
    // operands as one box of BK rows per 128-byte column block. Two rows per
    // stage halve the barrier handoffs and MMA commits per FLOP.
    static constexpr int KB = KB_;
    static constexpr int BK = KB * 128 / ES;
    static constexpr int MNBOX = 128 / ES;              // MN-major box width
    static constexpr int A_BYTES = BM * 128 * KB;
    static constexpr int BNL = PAIR ? BN / 2 : BN;     // B columns landed per CTA
    static constexpr int B_BYTES = BNL * 128 * KB;
    static constexpr int TX_BYTES = A_BYTES + B_BYTES;
    static constexpr int STAGE_BYTES = TX_BYTES * (F32 ? 2 : 1);
    // epilogue warps: 4 (one per TMEM lane quadrant) or more, sharing quadrants
    // by alternating 32-column chunks; more warps raise the output rate of
    // store-bound shapes. The epilogue uses no shared memory, so the operand
    // ring takes the whole 224 KB budget.
    static constexpr int EPIW = EPIW_;
    static constexpr int STAGES = (224 * 1024) / STAGE_BYTES;
    static constexpr int UMMA_K = F32 ? 8 : 16;
    static constexpr int KSUB = BK / UMMA_K;
    static constexpr int KSUB1 = 128 / ES / UMMA_K;     // MMA k-steps per 128-byte row
    // fp32: each accumulator buffer holds two BN-column sums (big*big and the
    // two cross terms), added with one IEEE fp32 add in the epilogue
    // TMEM holds 4 (fp32) or 2 (fp16) BN-column slots. fp16: two accumulator
    // buffers of one slot. fp32: the k-steps of a tile rotate over acc_slots
    // (S = 1, 2 or 4) slots that the epilogue adds with IEEE fp32 adds, and
    // 4 / S buffers alternate between tiles.
    static constexpr int SLOTS = (F32 && BN == 128) ? 4 : 2;
    static constexpr int TMEM_COLS = SLOTS * BN;
    // fp32: warps computing the tf32 small halves in shared memory (0 when
    // the variant is only used with both halves precomputed)
    static constexpr int SPLITW = SPLITW_;
    static constexpr int THREADS = 64 + 32 * EPIW + 32 * SPLITW;
    static constexpr int NBARS = 3 * STAGES + 9;
    static constexpr int SMEM = 1024 + STAGES * STAGE_BYTES + NBARS * 8 + 16;
    static_assert(SMEM <= 232448, "shared memory budget");
    static_assert(TMEM_COLS == 256 || TMEM_COLS == 512, "TMEM allocation must be a power of two");
    // fp32 pairs only with both tf32 small halves precomputed (no split warps)
    static_assert(!PAIR || !F32 || SPLITW == 0, "fp32 CTA pairs need precomputed small halves");
    static_assert(KB == 1 || !F32, "two-row stages are fp16 only");
};

// Batch coordinates of flat batch index i in one map (fully unrolled so the
// coordinates stay in registers).
__device__ __forceinline__ void batch_coords(const MapBatch& b, uint32_t i, int (&c)[3]) {
#pragma unroll
    for (int j = 0; j < kMaxBatchMap; ++j) c[j] = j < b.nb ? (int)((i / b.div[j]) % b.size[j]) : 0;
}

__device__ __forceinline__ int64_t decode_off(const Decode& d, int64_t x) {
    if (d.n == 1) return x * d.stride[0];
    int64_t off = 0;
    for (int a = d.n - 1; a >= 0; --a) {
        int64_t q = x / d.size[a];
        off += (x - q * d.size[a]) * d.stride[a];
        x = q;
    }
    return off;
}

// Bounded wait that ignores the abort flag: used only while draining.
__device__ __forceinline__ void drain_wait(uint32_t bar, uint32_t parity) {
    uint64_t t0 = globaltimer();
    while (!mbar_try_wait(bar, parity)) {
        if (globaltimer() - t0 > 200000000ull) {
            record_error(PE_ERR_TIMEOUT | (9 << 8));
            return;
        }
    }
}

// The idx-th work unit of CTA (group) `unit0` of `ustep`: output tile t, its
// k-iteration range [kb_lo, kb_hi) and the partial slab sp it writes.
// Split-K (sk_q == 0): units are (tile, equal k-slice) pairs dealt round-robin.
// Stream-K (sk_q > 0): CTA c owns the flattened iterations [c*Q, (c+1)*Q) of
// the (tile, k) space and emits one partial per tile it touches; sp numbers the
// segments of a tile by the CTA boundaries inside it, so a deterministic
// reduction can sum them in order.
__device__ __forceinline__ bool work_unit(const GemmArgs& g, int unit0, int ustep, int idx, int& t, int& sp,
                                          int& kb_lo, int& kb_hi) {
    if (g.sk_q > 0) {
        const int64_t q = g.sk_q;
        const int64_t lo = (int64_t)unit0 * q;
        const int64_t hi = min(lo + q, (int64_t)g.tiles * g.kiters);
        const int64_t tt = lo / g.kiters + idx;
        const int64_t base = tt * g.kiters;
        if (base >= hi) return false;
        t = (int)tt;
        kb_lo = (int)(lo > base ? lo - base : 0);
        kb_hi = (int)min(hi - base, (int64_t)g.kiters);
        sp = (int)((base + kb_lo) / q - base / q);
        return true;
    }
    const int u = unit0 + idx * ustep;
    if (u >= g.tiles * g.ksplit) return false;
    t = u / g.ksplit;
    sp = u - t * g.ksplit;
    kb_lo = sp * g.kper;
    kb_hi = min(g.kiters, kb_lo + g.kper);
    return true;
}

// Diagnostic build (-DPE_STALL_STATS): per-CTA cycle counts of each pipeline
// role's waits, read back with pe_stall_stats(). Slots: 0 producer waiting for a
// free stage, 1 MMA thread waiting for landed operands, 2 MMA thread waiting for
// a drained accumulator, 3 epilogue warp 2 waiting for a finished accumulator,
// 4 epilogue warp 2 busy (accumulator ready -> handed back), 5 kernel cycles
// (thread 0), 6 tiles.
#ifdef PE_STALL_STATS
__device__ unsigned long long pe_stall[1024 * 8];
#define PE_STALL_BEGIN() const long long _st0 = clock64()
#define PE_STALL_END(slot) atomicAdd(&pe_stall[blockIdx.x * 8 + (slot)], (unsigned long long)(clock64() - _st0))
#define PE_STALL_ADD(slot, v) atomicAdd(&pe_stall[blockIdx.x * 8 + (slot)], (unsigned long long)(v))
#else
#define PE_STALL_BEGIN() ((void)0)
#define PE_STALL_END(slot) ((void)0)
#define PE_STALL_ADD(slot, v) ((void)0)
#endif

template <class C>
__global__ void __launch_bounds__(C::THREADS, 1) gemm_kernel(const __grid_constant__ GemmArgs g) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint64_t* bars = (uint64_t*)(smem + C::STAGES * C::STAGE_BYTES);
    uint32_t* tmem_slot = (uint32_t*)(bars + C::NBARS);
    volatile int* abort_flag = (volatile int*)(tmem_slot + 1);

    const uint32_t bar0 = smem_u32(bars);
    auto full = [&](int s) { return bar0 + 8u * s; };
    auto empty = [&](int s) { return bar0 + 8u * (C::STAGES + s); };
    auto split = [&](int s) { return bar0 + 8u * (2 * C::STAGES + s); };
    auto tfull = [&](int a) { return bar0 + 8u * (3 * C::STAGES + a); };
    auto tempty = [&](int a) { return bar0 + 8u * (3 * C::STAGES + 4 + a); };
    const uint32_t mma_done = bar0 + 8u * (3 * C::STAGES + 8);
    const int S = C::F32 ? g.acc_slots : 1;     // accumulator slots per tile
    const bool split_done_by_tma = g.a_pre && g.b_pre;  // fp32: both small halves precomputed
    const int NBUF = C::SLOTS / S;              // accumulator buffers

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = C::PAIR ? cluster_rank() : 0;        // CTA rank in the pair
    const int unit0 = C::PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
    const int ustep = C::PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;
    if (threadIdx.x == 0) {
        for (int s = 0; s < C::STAGES; ++s) {
            mbar_init(full(s), 1);
            mbar_init(empty(s), 1);
            mbar_init(split(s), 128);
        }
        for (int a = 0; a < 4; ++a) {
            mbar_init(tfull(a), 1);
            mbar_init(tempty(a), C::PAIR ? 2 * C::EPIW : C::EPIW);
        }
        mbar_init(mma_done, 1);
        *abort_flag = 0;
        fence_barrier_init();
        tma_prefetch(&g.tma);
        tma_prefetch(&g.tmb);
    }
    if (warp == 1) {
        if constexpr (C::PAIR) {
            tmem_alloc_pair(smem_u32(tmem_slot), C::TMEM_COLS);
            tmem_relinquish_pair();
        } else {
            tmem_alloc(smem_u32(tmem_slot), C::TMEM_COLS);
            tmem_relinquish();
        }
        tc_fence_before();
    }
    __syncthreads();
    if constexpr (C::PAIR) cluster_sync();  // barrier inits visible to the peer CTA
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const int per_batch = g.mblk * g.nblk;
    // Programmatic dependent launch: the prologue above (barrier init, TMEM
    // allocation, descriptor prefetch) overlaps the previous kernel's tail; no
    // global memory is read or written before the previous grid has finished.
    // Dependents are released at once: they only become resident as this
    // grid's CTAs exit, and they wait the same way.
    grid_dep_wait();
    grid_dep_launch();
#ifdef PE_STALL_STATS
    const long long k_t0 = clock64();
#endif

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer ----------------
            int stage = 0;
            uint32_t phase = 0;
            uint32_t issued_mask = 0, issued_par = 0;
            int t, sp, kb_lo, kb_hi;
            for (int idx = 0; !*abort_flag && work_unit(g, unit0, ustep, idx, t, sp, kb_lo, kb_hi); ++idx) {
                const int i = t / per_batch, r = t - i * per_batch;
                const int m0 = (r / g.nblk) * C::TM + (int)rank * C::BM;   // this CTA's A rows
                const int n0 = (r % g.nblk) * C::BN + (int)rank * (C::BN - C::BNL);  // its B columns
                int ca[3], cb[3];
                batch_coords(g.ab, i, ca);
                batch_coords(g.bb, i, cb);
                for (int kb = kb_lo; kb < kb_hi; ++kb) {
                    PE_STALL_BEGIN();
                    if (!mbar_wait(empty(stage), phase ^ 1, abort_flag, 1)) break;
                    PE_STALL_END(0);
                    uint8_t* sa = smem + stage * C::STAGE_BYTES;
                    uint8_t* sb = sa + C::A_BYTES;
                    const int k0 = kb * C::BK;
                    // pairs: the leader's barrier counts both CTAs' bytes
                    int tx = C::TX_BYTES;
                    if constexpr (C::F32) tx += (g.a_pre ? C::A_BYTES : 0) + (g.b_pre ? C::B_BYTES : 0);
                    if constexpr (C::PAIR) tx *= 2;
                    if (g.phase < 1) {
                        // phase gate: the stage completes without data
                        if (rank == 0) mbar_arrive(full(stage));
                        if (++stage == C::STAGES) {
                            stage = 0;
                            phase ^= 1;
                        }
                        continue;
                    }
                    if (rank == 0) mbar_arrive_expect_tx(full(stage), tx);
                    issued_mask |= 1u << stage;
                    issued_par = (issued_par & ~(1u << stage)) | (phase << stage);
                    auto load = [&](uint32_t dst, const CUtensorMap* tm, int x0, int x1, const int (&c)[3]) {
                        if constexpr (C::PAIR)
                            tma_load_5d_pair(dst, tm, full(stage), x0, x1, c[0], c[1], c[2]);
                        else
                            tma_load_5d(dst, tm, full(stage), x0, x1, c[0], c[1], c[2]);
                    };
                    auto load_a = [&](uint8_t* dst, const CUtensorMap* tm) {
                        if (!g.a_mn) {
#pragma unroll
                            for (int u = 0; u < C::KB; ++u)
                                load(smem_u32(dst + u * C::BM * 128), tm, k0 + u * C::MNBOX, m0, ca);
                        } else {
#pragma unroll
                            for (int j = 0; j < C::BM / C::MNBOX; ++j)
                                load(smem_u32(dst + j * C::BK * 128), tm, m0 + j * C::MNBOX, k0, ca);
                        }
                    };
                    auto load_b = [&](uint8_t* dst, const CUtensorMap* tm) {
                        if (!g.b_mn) {
#pragma unroll
                            for (int u = 0; u < C::KB; ++u)
                                load(smem_u32(dst + u * C::BNL * 128), tm, k0 + u * C::MNBOX, n0, cb);
                        } else {
#pragma unroll
                            for (int j = 0; j < C::BNL / C::MNBOX; ++j)
                                load(smem_u32(dst + j * C::BK * 128), tm, n0 + j * C::MNBOX, k0, cb);
                        }
                    };
                    load_a(sa, &g.tma);
                    load_b(sb, &g.tmb);
                    if constexpr (C::F32) {
                        // fused-B stages: [A][B][B small][A small]
                        if (g.a_pre) load_a(sa + C::TX_BYTES + (g.fuse_b ? C::B_BYTES : 0), &g.tmas);
                        if (g.b_pre) load_b(g.fuse_b ? sb + C::B_BYTES : sb + C::TX_BYTES, &g.tmbs);
                    }
                    if (++stage == C::STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
            if (*abort_flag && rank == 0) {
                // let every load still in flight land before shared memory is released
                // (pairs: the leader's barriers also count the peer's loads)
                for (int s = 0; s < C::STAGES; ++s)
                    if (issued_mask & (1u << s)) drain_wait(full(s), (issued_par >> s) & 1);
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && rank == 0) {
            // ---------------- MMA issuer (pairs: the leader CTA only) ----------------
            const uint32_t idesc = make_idesc(C::F32 ? 2u : 0u, C::TM, C::BN, g.a_mn, g.b_mn);
            const uint32_t idesc2 = make_idesc(2u, C::TM, 2 * C::BN, g.a_mn, g.b_mn);  // fused B: N = 2 BN
            // byte step of one UMMA_K slice and leading offsets of MN-major tiles
            const uint32_t a_kstep = g.a_mn ? (C::UMMA_K / 8) * 1024 : 32;
            const uint32_t b_kstep = g.b_mn ? (C::UMMA_K / 8) * 1024 : 32;
            const uint32_t a_lbo = g.a_mn ? C::BK * 128 : 16;
            const uint32_t b_lbo = g.b_mn ? C::BK * 128 : 16;
            // MN-major tf32 tiles use the 128B swizzle with 32-byte atoms (swizzle
            // period 4 rows): layout type 1 and a 512-byte k-group stride.
            const uint32_t a_lay = (C::F32 && g.a_mn) ? 1u : 2u, b_lay = (C::F32 && g.b_mn) ? 1u : 2u;
            const uint32_t a_sbo = a_lay == 1 ? 512 : 1024, b_sbo = b_lay == 1 ? 512 : 1024;
            int stage = 0, acc = 0;
            uint32_t phase = 0, acc_phase = 0;
            int t, sp, kb_lo, kb_hi;
            for (int idx = 0; !*abort_flag && work_unit(g, unit0, ustep, idx, t, sp, kb_lo, kb_hi); ++idx) {
                {
                    PE_STALL_BEGIN();
                    if (!mbar_wait(tempty(acc), acc_phase ^ 1, abort_flag, 2)) break;
                    PE_STALL_END(2);
                }
                tc_fence_after();
                const uint32_t dbuf = tmem_base + (uint32_t)(acc * S * C::BN);
                bool ok = true;
                for (int kb = kb_lo; kb < kb_hi; ++kb) {
                    PE_STALL_BEGIN();
                    if (!mbar_wait(C::F32 && !split_done_by_tma ? split(stage) : full(stage), phase, abort_flag, 3)) {
                        ok = false;
                        break;
                    }
                    PE_STALL_END(1);
                    tc_fence_after();
                    const uint32_t sa = smem_u32(smem + stage * C::STAGE_BYTES);
                    const uint32_t sb = sa + C::A_BYTES;
                    const int slot = C::F32 ? (kb - kb_lo) % S : 0;
                    const uint32_t d = dbuf + (uint32_t)(slot * C::BN);
#pragma unroll
                    for (int ks = 0; ks < C::KSUB; ++ks) {
                        if (g.phase < 2) break;  // phase gate: no MMAs
                        // K-major: k-step ks lies in row block ks / KSUB1 of the stage
                        const uint32_t a_off = g.a_mn ? ks * a_kstep
                                                      : (ks / C::KSUB1) * (C::BM * 128) + (ks % C::KSUB1) * a_kstep;
                        const uint32_t b_off = g.b_mn ? ks * b_kstep
                                                      : (ks / C::KSUB1) * (C::BNL * 128) + (ks % C::KSUB1) * b_kstep;
                        const uint64_t ad = smem_desc_sw128(sa + a_off, a_lbo, a_sbo, a_lay);
                        const uint64_t bd = smem_desc_sw128(sb + b_off, b_lbo, b_sbo, b_lay);
                        const uint32_t accum = (kb - kb_lo >= S || ks > 0) ? 1u : 0u;
                        if constexpr (C::F32 && !C::PAIR && C::BN == 128) {
                            if (g.fuse_b) {
                                // [Bb | Bs] is one 256-column operand (Bs follows B in the
                                // stage with the same layout): D1 = Ab.Bb, D2 = Ab.Bs, then
                                // D2 += As.Bb; k-steps alternate between two (D1, D2) pairs
                                const uint64_t ads = smem_desc_sw128(sa + C::TX_BYTES + C::B_BYTES + ks * a_kstep, a_lbo,
                                                                     a_sbo, a_lay);
                                const uint32_t dd = dbuf + (uint32_t)(((kb - kb_lo) & 1) * 2 * C::BN);
                                const uint32_t acc1 = (kb - kb_lo >= 2 || ks > 0) ? 1u : 0u;
                                mma_tf32(dd, ad, bd, idesc2, acc1);
                                mma_tf32(dd + C::BN, ads, bd, idesc, 1u);
                                continue;
                            }
                        }
                        if constexpr (C::F32) {
                            const uint64_t ads = smem_desc_sw128(sa + C::TX_BYTES + ks * a_kstep, a_lbo, a_sbo, a_lay);
                            const uint64_t bds = smem_desc_sw128(sb + C::TX_BYTES + ks * b_kstep, b_lbo, b_sbo, b_lay);
                            if constexpr (C::PAIR) {
                                mma_tf32_pair(d, ads, bd, idesc, accum);
                                mma_tf32_pair(d, ad, bds, idesc, 1u);
                                mma_tf32_pair(d, ad, bd, idesc, 1u);
                            } else {
                                mma_tf32(d, ads, bd, idesc, accum);
                                mma_tf32(d, ad, bds, idesc, 1u);
                                mma_tf32(d, ad, bd, idesc, 1u);
                            }
                        } else if constexpr (C::PAIR) {
                            mma_f16_pair(d, ad, bd, idesc, accum);
                        } else {
                            mma_f16(d, ad, bd, idesc, accum);
                        }
                    }
                    if constexpr (C::PAIR) mma_commit_pair_mc(empty(stage), 0x3);
                    else mma_commit(empty(stage));
                    if (++stage == C::STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
                if (!ok) break;
                if constexpr (C::PAIR) mma_commit_pair_mc(tfull(acc), 0x3);
                else mma_commit(tfull(acc));
                if (++acc == NBUF) {
                    acc = 0;
                    acc_phase ^= 1;
                }
            }
            // all MMAs issued by this thread complete before TMEM is released
            if constexpr (C::PAIR) mma_commit_pair(mma_done);
            else mma_commit(mma_done);
            drain_wait(mma_done, 0);
        }
    } else if (warp < 2 + C::EPIW) {
        // ---------------- epilogue: TMEM -> registers -> global ----------------
        // Warp w may only read TMEM lanes 32*(w%4)..+31, so the warps sharing a
        // lane quadrant take alternate 32-column chunks of the tile. The next
        // chunk's tcgen05.ld is issued before the current chunk is staged
        // and stored, hiding the TMEM load latency.
        constexpr int NH = C::EPIW / 4;
        const int ew = warp - 2;
        const int q = warp & 3;
        const int half = ew >> 2;
        int acc = 0;
        uint32_t acc_phase = 0;
        int t, sp, kb_lo, kb_hi;
        for (int idx = 0; !*abort_flag && work_unit(g, unit0, ustep, idx, t, sp, kb_lo, kb_hi); ++idx) {
            const int i = t / per_batch, r = t - i * per_batch;
            const int m0 = (r / g.nblk) * C::TM + (int)rank * C::BM, n0 = (r % g.nblk) * C::BN;
#ifdef PE_STALL_STATS
            const long long e_t0 = clock64();
#endif
            if (!mbar_wait(tfull(acc), acc_phase, abort_flag, 4)) break;
#ifdef PE_STALL_STATS
            const long long e_t1 = clock64();
            if (ew == 0 && lane == 0) {
                PE_STALL_ADD(3, e_t1 - e_t0);
                PE_STALL_ADD(6, 1);
            }
#endif
            tc_fence_after();
            const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * S * C::BN);
            // fused B: two 128-column halves per k-rotation slot, up to two slots
            const int nslots = g.fuse_b ? 2 * min(2, kb_hi - kb_lo) : (S < kb_hi - kb_lo ? S : kb_hi - kb_lo);
            const int bidx = i + sp * g.nbatch;  // output batch (split-K: partial slab sp)
            const int mrow = m0 + q * 32;
            const int m = mrow + lane;
            const int nvalid = min(C::BN / 32, (g.N - n0 + 31) / 32);
            int64_t row_off = 0;
            if (m < g.M) row_off = decode_off(g.ob, bidx) + decode_off(g.om, m);
            // unit-stride outputs: row offsets are affine in the row index
            const int64_t row_base = decode_off(g.ob, bidx);
            const int64_t mst = g.om.stride[0];
            // Strided outputs: sum the accumulator slots (fp32) and write one
            // 32x32 chunk held as lane = row, v[j] = column nc + j, each element
            // to its decoded offset.
            auto emit = [&](uint32_t (&v)[32], int c) {
                const int nc = n0 + c * 32;
                if constexpr (C::F32) {
                    for (int sl = 1; sl < nslots; ++sl) {
                        uint32_t w[32];
                        __syncwarp();
                        tmem_ld32(tbase + (uint32_t)(sl * C::BN) + c * 32, w);
                        tmem_ld_wait();
#pragma unroll
                        for (int j = 0; j < 32; ++j)
                            v[j] = __float_as_uint(__uint_as_float(v[j]) + __uint_as_float(w[j]));
                    }
                }
                if (m < g.M) {
                    float* o = g.out + row_off;
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        const int n = nc + j;
                        if (n < g.N) o[decode_off(g.on, n)] = __uint_as_float(v[j]);
                    }
                }
            };
            const int nv = g.phase >= 3 ? nvalid : 0;  // phase gate: no TMEM reads or stores
            if (g.out_rows) {
                // Unit-stride rows: each 16-lane half of the warp's quadrant is
                // read in the 16x256b layout, where four threads hold 8 consecutive
                // columns (one 32-byte sector) of one row, so every 8-byte store
                // instruction writes 8 full sectors straight from registers. (A
                // 32x32b read transposed through swizzled shared memory into 16-byte
                // stores covering four 128-byte row pieces was measured first: the
                // staging traffic competed with the operand pipeline for the
                // shared-memory port and output-bound shapes ran 5-10% slower.)
                auto load_chunk = [&](uint32_t (&r)[2][16], int c) {
                    tmem_ld16x256_x4(tbase + c * 32, r[0]);
                    tmem_ld16x256_x4(tbase + (16u << 16) + c * 32, r[1]);
                };
                auto store_chunk = [&](uint32_t (&r)[2][16], int c) {
                    const int nc = n0 + c * 32;
                    if constexpr (C::F32) {
                        for (int sl = 1; sl < nslots; ++sl) {
#pragma unroll
                            for (int h = 0; h < 2; ++h) {
                                uint32_t w[16];
                                __syncwarp();
                                tmem_ld16x256_x4(tbase + ((uint32_t)(16 * h) << 16) + (uint32_t)(sl * C::BN) + c * 32, w);
                                tmem_ld_wait();
#pragma unroll
                                for (int j = 0; j < 16; ++j)
                                    r[h][j] = __float_as_uint(__uint_as_float(r[h][j]) + __uint_as_float(w[j]));
                            }
                        }
                    }
                    if (g.out_v8) {
                        // The four lanes of a quad hold one row: lane q has the column
                        // pairs 8j + 2q (j = 0..3). A two-stage butterfly (xor 1, then
                        // xor 2) transposes the 4x4 pair matrix so that lane q holds
                        // columns 8q..8q+7, and one 32-byte store per lane writes the
                        // row's 128 bytes: eight full lines per warp instruction instead
                        // of eight 32-byte sectors.
                        const bool ql = lane & 1, qh = (lane >> 1) & 1;
#pragma unroll
                        for (int h = 0; h < 2; ++h) {
#pragma unroll
                            for (int rr = 0; rr < 2; ++rr) {
                                uint32_t e[4][2], f[2][2][2], o[4][2];
#pragma unroll
                                for (int j = 0; j < 4; ++j) {
                                    e[j][0] = r[h][4 * j + 2 * rr];
                                    e[j][1] = r[h][4 * j + 2 * rr + 1];
                                }
                                // stage 1: keep the pair with j's low bit = ql, swap the other
#pragma unroll
                                for (int jh = 0; jh < 2; ++jh) {
#pragma unroll
                                    for (int w = 0; w < 2; ++w) {
                                        const uint32_t send = ql ? e[2 * jh][w] : e[2 * jh + 1][w];
                                        const uint32_t keep = ql ? e[2 * jh + 1][w] : e[2 * jh][w];
                                        const uint32_t recv = __shfl_xor_sync(0xffffffffu, send, 1);
                                        f[jh][0][w] = ql ? recv : keep;
                                        f[jh][1][w] = ql ? keep : recv;
                                    }
                                }
                                // stage 2: keep jh = qh, swap the other
#pragma unroll
                                for (int rl = 0; rl < 2; ++rl) {
#pragma unroll
                                    for (int w = 0; w < 2; ++w) {
                                        const uint32_t send = qh ? f[0][rl][w] : f[1][rl][w];
                                        const uint32_t keep = qh ? f[1][rl][w] : f[0][rl][w];
                                        const uint32_t recv = __shfl_xor_sync(0xffffffffu, send, 2);
                                        o[rl][w] = qh ? recv : keep;
                                        o[2 + rl][w] = qh ? keep : recv;
                                    }
                                }
                                const int row = mrow + 16 * h + 8 * rr + (lane >> 2);
                                if (row >= g.M) continue;
                                float* dst = g.out + row_base + (int64_t)row * mst;
                                const int n = nc + 8 * (lane & 3);
                                if (n + 8 <= g.N) {
                                    st_global_v8(dst + n, o);
                                } else {
#pragma unroll
                                    for (int j = 0; j < 8; ++j)
                                        if (n + j < g.N) dst[n + j] = __uint_as_float(o[j >> 1][j & 1]);
                                }
                            }
                        }
                        return;
                    }
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
#pragma unroll
                        for (int rr = 0; rr < 2; ++rr) {
                            const int row = mrow + 16 * h + 8 * rr + (lane >> 2);
                            if (row >= g.M) continue;
                            float* dst = g.out + row_base + (int64_t)row * mst;
#pragma unroll
                            for (int j = 0; j < 4; ++j) {
                                const int n = nc + 8 * j + 2 * (lane & 3);
                                const uint32_t x = r[h][4 * j + 2 * rr], y = r[h][4 * j + 2 * rr + 1];
                                if (n + 2 <= g.N) {
                                    *reinterpret_cast<uint2*>(dst + n) = make_uint2(x, y);
                                } else if (n < g.N) {
                                    dst[n] = __uint_as_float(x);
                                }
                            }
                        }
                    }
                };
                // One register buffer: measured against two (the next chunk's TMEM
                // reads in flight while the current chunk is stored), which spilled
                // and ran 10-15% slower on the output-bound configs.
                uint32_t ra[2][16];
                for (int c = half; c < nv; c += NH) {
                    __syncwarp();
                    load_chunk(ra, c);
                    tmem_ld_wait();
                    store_chunk(ra, c);
                }
            }
            // Two register buffers: the TMEM load of the next chunk is in flight
            // while the current one is written out.
            uint32_t va[32], vb[32];
            if (half < nv && !g.out_rows) {
                __syncwarp();
                tmem_ld32(tbase + half * 32, va);
                tmem_ld_wait();
            }
#pragma unroll 1
            for (int c = half; c < (g.out_rows ? 0 : nv); c += 2 * NH) {
                const int c1 = c + NH, c2 = c + 2 * NH;
                __syncwarp();
                if (c1 < nv) tmem_ld32(tbase + c1 * 32, vb);
                emit(va, c);
                if (c1 >= nv) break;
                __syncwarp();
                tmem_ld_wait();
                if (c2 < nv) tmem_ld32(tbase + c2 * 32, va);
                emit(vb, c1);
                __syncwarp();
                if (c2 < nv) tmem_ld_wait();
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                if constexpr (C::PAIR) mbar_arrive_cluster(map_to_rank(tempty(acc), 0));  // leader's barrier
                else mbar_arrive(tempty(acc));
#ifdef PE_STALL_STATS
                if (ew == 0) PE_STALL_ADD(4, clock64() - e_t1);
#endif
            }
            if (++acc == NBUF) {
                acc = 0;
                acc_phase ^= 1;
            }
        }
    } else if constexpr (C::F32 && C::SPLITW == 4) {
        // ---------------- 3xTF32 split: x -> big (in place) + small ----------------
        const int st = threadIdx.x - 32 * (2 + C::EPIW);
        // 16-byte pieces to split this stage: operands whose small half was
        // precomputed arrive with it and are skipped
        const int jlo = g.a_pre ? C::A_BYTES / 16 : 0;
        const int jhi = g.b_pre ? C::A_BYTES / 16 : C::TX_BYTES / 16;
        int stage = 0;
        uint32_t phase = 0;
        int t, sp, kb_lo, kb_hi;
        for (int idx = 0; !split_done_by_tma && !*abort_flag && work_unit(g, unit0, ustep, idx, t, sp, kb_lo, kb_hi);
             ++idx) {
            bool ok = true;
            for (int kb = kb_lo; kb < kb_hi; ++kb) {
                if (!mbar_wait(full(stage), phase, abort_flag, 5)) {
                    ok = false;
                    break;
                }
                uint4* big = reinterpret_cast<uint4*>(smem + stage * C::STAGE_BYTES);
                // small halves mirror [A][B] at TX_BYTES; fused-B stages hold [B small][A small]
                uint4* small_a = reinterpret_cast<uint4*>(smem + stage * C::STAGE_BYTES + C::TX_BYTES +
                                                          (g.fuse_b ? C::B_BYTES : 0));
                uint4* small_b = reinterpret_cast<uint4*>(smem + stage * C::STAGE_BYTES + C::TX_BYTES -
                                                          (g.fuse_b ? C::A_BYTES : 0));
#pragma unroll 4
                for (int j = jlo + st; j < jhi; j += 128) {
                    uint4 x = big[j];
                    uint4 h = make_uint4(x.x & 0xFFFFE000u, x.y & 0xFFFFE000u, x.z & 0xFFFFE000u,
                                         x.w & 0xFFFFE000u);
                    float4 s = make_float4(__uint_as_float(x.x) - __uint_as_float(h.x),
                                           __uint_as_float(x.y) - __uint_as_float(h.y),
                                           __uint_as_float(x.z) - __uint_as_float(h.z),
                                           __uint_as_float(x.w) - __uint_as_float(h.w));
                    if (!g.raw_big) big[j] = h;
                    (j < C::A_BYTES / 16 ? small_a : small_b)[j] = *reinterpret_cast<uint4*>(&s);
                }
                fence_proxy_async_smem();
                mbar_arrive(split(stage));
                if (++stage == C::STAGES) {
                    stage = 0;
                    phase ^= 1;
                }
            }
            if (!ok) break;
        }
    }

    __syncthreads();
#ifdef PE_STALL_STATS
    if (threadIdx.x == 0) PE_STALL_ADD(5, clock64() - k_t0);
#endif
    // pairs: the leader's MMAs write the peer's TMEM and both CTAs' barriers
    // receive remote arrivals, so neither CTA leaves before the other is done
    if constexpr (C::PAIR) cluster_sync();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        if constexpr (C::PAIR) tmem_dealloc_pair(tmem_base, C::TMEM_COLS);
        else tmem_dealloc(tmem_base, C::TMEM_COLS);
    }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------

PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (PFN_cuTensorMapEncodeTiled_v12000)p;
    });
    return fn;
}

struct Axis {
    int64_t size, stride;
};

// Drop size-1 axes and merge neighbours that are contiguous in memory
// (outer.stride == inner.stride * inner.size). Axes are outermost first.
int coalesce(const Axis* in, int n, Axis* out) {
    int k = 0;
    for (int a = 0; a < n; ++a) {
        if (in[a].size == 1) continue;
        if (k > 0 && out[k - 1].stride == in[a].stride * in[a].size) {
            out[k - 1].size *= in[a].size;
            out[k - 1].stride = in[a].stride;
        } else {
            out[k++] = in[a];
        }
    }
    return k;
}

// Joint coalescing of the batch axes of one map: batch index order is kept.
struct OperandView {
    bool direct = false;
    bool mn_major = false;
    const void* base = nullptr;
    int64_t mn_size = 1, mn_stride = 0, k_size = 1, k_stride = 0;
    int nb = 0;
    int64_t b_size[kMaxBatchMap] = {1, 1, 1}, b_stride[kMaxBatchMap] = {0, 0, 0};
};

inline bool al16(int64_t bytes) { return (bytes & 15) == 0; }

// Describe one operand (axes already split into batch / free / contract groups)
// as a tensor-map-readable view, if possible.
OperandView view_direct(const void* base, int es, const Axis* batch, int nb, const Axis* fr, int nf,
                        const Axis* ct, int nc) {
    OperandView v;
    v.base = base;
    if (((uintptr_t)base & 15) != 0) return v;
    Axis m[PE_MAX_RANK], k[PE_MAX_RANK], b[PE_MAX_RANK];
    int nm = coalesce(fr, nf, m), nk = coalesce(ct, nc, k), nbb = coalesce(batch, nb, b);
    if (nm > 1 || nk > 1 || nbb > kMaxBatchMap) return v;
    if (nm == 1) { v.mn_size = m[0].size; v.mn_stride = m[0].stride; }
    if (nk == 1) { v.k_size = k[0].size; v.k_stride = k[0].stride; }
    for (int j = 0; j < nbb; ++j) {
        if (!al16(b[j].stride * es)) return v;
        v.b_size[j] = b[j].size;
        v.b_stride[j] = b[j].stride;
    }
    v.nb = nbb;
    const bool k_unit = v.k_size == 1 || v.k_stride == 1;
    const bool m_unit = v.mn_size == 1 || v.mn_stride == 1;
    const bool m_al = v.mn_size == 1 || al16(v.mn_stride * es);
    const bool k_al = v.k_size == 1 || al16(v.k_stride * es);
    if (k_unit && m_al) {
        v.mn_major = false;
    } else if (m_unit && k_al) {
        v.mn_major = true;
    } else {
        return v;
    }
    if (v.mn_size > 0xFFFFFFFFll || v.k_size > 0xFFFFFFFFll) return v;
    v.direct = true;
    return v;
}

// Rank-5 tensor map of an operand view: dims {inner, outer, batch0..2}.
bool encode_operand(CUtensorMap* tm, const OperandView& v, bool f32, int box_mn_rows, int box_k_rows = 0) {
    auto enc = get_encode();
    if (!enc) return false;
    const int es = f32 ? 4 : 2;
    cuuint64_t dims[5];
    cuuint64_t strides[4];
    cuuint32_t box[5] = {0, 0, 1, 1, 1};
    cuuint32_t estr[5] = {1, 1, 1, 1, 1};
    const int bk = 128 / es;
    if (!v.mn_major) {
        dims[0] = (cuuint64_t)v.k_size;
        dims[1] = (cuuint64_t)v.mn_size;
        strides[0] = (cuuint64_t)((v.mn_size == 1 ? 1 : v.mn_stride) * es);
        box[0] = bk;
        box[1] = box_mn_rows;
    } else {
        dims[0] = (cuuint64_t)v.mn_size;
        dims[1] = (cuuint64_t)v.k_size;
        strides[0] = (cuuint64_t)((v.k_size == 1 ? 1 : v.k_stride) * es);
        box[0] = bk;
        box[1] = box_k_rows > 0 ? box_k_rows : bk;
    }
    int64_t ext = 16;  // any valid stride for padded size-1 dims
    for (int j = 0; j < kMaxBatchMap; ++j) {
        dims[2 + j] = (cuuint64_t)(j < v.nb ? v.b_size[j] : 1);
        if (j < v.nb) {
            strides[1 + j] = (cuuint64_t)(v.b_stride[j] * es);
            int64_t e = v.b_stride[j] * es * v.b_size[j];
            if (e > ext) ext = e;
        }
    }
    {
        int64_t e = (int64_t)strides[0] * (int64_t)dims[1];
        if (e > ext) ext = e;
    }
    ext = (ext + 15) & ~(int64_t)15;
    for (int j = v.nb; j < kMaxBatchMap; ++j) strides[1 + j] = (cuuint64_t)ext;
    // size-1 outer dim: its stride is unused, make it valid
    if (dims[1] == 1) strides[0] = (cuuint64_t)ext;
    for (int j = 0; j < 4; ++j)
        if ((strides[j] & 15) || strides[j] >= (1ull << 40)) return false;
    CUresult r = enc(tm, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 5,
                     const_cast<void*>(v.base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE,
                     (f32 && v.mn_major) ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

MapBatch map_batch(const OperandView& v) {
    MapBatch b{};
    b.nb = v.nb;
    uint64_t run = 1;
    for (int j = v.nb - 1; j >= 0; --j) {
        b.size[j] = (uint32_t)v.b_size[j];
        b.div[j] = (uint32_t)run;
        run *= (uint64_t)v.b_size[j];
    }
    return b;
}

// Output: interp axes (batch, free0, free1) with strides of the permuted output.
struct OutView {
    Axis b[PE_MAX_RANK], m[PE_MAX_RANK], n[PE_MAX_RANK];
    int nb, nm, nn;
};

bool encode_output(CUtensorMap* tm, float* out, const OutView& o, MapBatch* mb) {
    auto enc = get_encode();
    if (!enc || ((uintptr_t)out & 15)) return false;
    Axis m[PE_MAX_RANK], n[PE_MAX_RANK], b[PE_MAX_RANK];
    int nm = coalesce(o.m, o.nm, m), nn = coalesce(o.n, o.nn, n), nbb = coalesce(o.b, o.nb, b);
    if (nm > 1 || nn > 1 || nbb > kMaxBatchMap) return false;
    if (nn == 1 && n[0].stride != 1) return false;
    if (nm == 1 && !al16(m[0].stride * 4)) return false;
    cuuint64_t dims[5] = {(cuuint64_t)(nn ? n[0].size : 1), (cuuint64_t)(nm ? m[0].size : 1), 1, 1, 1};
    cuuint64_t strides[4];
    int64_t ext = 16;
    strides[0] = (cuuint64_t)(nm ? m[0].stride * 4 : 16);
    ext = std::max<int64_t>(ext, (int64_t)strides[0] * (int64_t)dims[1]);
    OperandView tmp;
    tmp.nb = nbb;
    for (int j = 0; j < nbb; ++j) {
        if (!al16(b[j].stride * 4)) return false;
        dims[2 + j] = (cuuint64_t)b[j].size;
        strides[1 + j] = (cuuint64_t)(b[j].stride * 4);
        ext = std::max<int64_t>(ext, b[j].stride * 4 * b[j].size);
        tmp.b_size[j] = b[j].size;
    }
    ext = (ext + 15) & ~(int64_t)15;
    for (int j = nbb; j < kMaxBatchMap; ++j) strides[1 + j] = (cuuint64_t)ext;
    if (dims[1] == 1) strides[0] = (cuuint64_t)ext;
    for (int j = 0; j < 4; ++j)
        if ((strides[j] & 15) || strides[j] >= (1ull << 40)) return false;
    cuuint32_t box[5] = {32, 32, 1, 1, 1};
    cuuint32_t estr[5] = {1, 1, 1, 1, 1};
    CUresult r = enc(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 5, out, dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return false;
    *mb = map_batch(tmp);
    return true;
}

// Every output row starts on a 32-byte boundary: base and the row and batch
// strides (elements) multiples of 8.
bool rows_aligned32(const float* out, const OutView& o) {
    if ((uintptr_t)out & 31) return false;
    for (int j = 0; j < o.nm; ++j)
        if (o.m[j].size > 1 && (o.m[j].stride & 7)) return false;
    for (int j = 0; j < o.nb; ++j)
        if (o.b[j].size > 1 && (o.b[j].stride & 7)) return false;
    return true;
}

// Full-line epilogue stores: on by default (output-bound shapes gained 2-6%,
// fp32 pairs included), off for fp16 CTA pairs (3% slower there: that
// mainloop is operand-load bound and the shuffles lengthen the epilogue). PE_EPI_V8=0/1
// forces either.
int epi_v8_enabled(bool fp16_pair) {
    const char* e = getenv("PE_EPI_V8");
    if (e && (e[0] == '0' || e[0] == '1')) return e[0] - '0';
    return fp16_pair ? 0 : 1;
}

Decode make_decode(const Axis* ax, int n) {
    Decode d{};
    Axis c[PE_MAX_RANK];
    int k = coalesce(ax, n, c);
    if (k == 0) {
        d.n = 1;
        d.size[0] = 1;
        d.stride[0] = 0;
        return d;
    }
    d.n = k;
    for (int a = 0; a < k; ++a) {
        d.size[a] = c[a].size;
        d.stride[a] = c[a].stride;
    }
    return d;
}

// Diagnostic: PE_GEMM_GRID_CAP=n runs the persistent grid on at most n SMs
// (used to tell a per-SM latency limit from a shared-bandwidth limit).
static int grid_cap() {
    static int cap = -1;
    if (cap < 0) {
        const char* e = getenv("PE_GEMM_GRID_CAP");
        const int v = e ? atoi(e) : 0;
        cap = (v > 0 && v < num_sms()) ? v : num_sms();
    }
    return cap;
}

// PE_GEMM_PDL=0 launches without programmatic dependent launch.
int pdl_enabled() {
    static int on = -1;
    if (on < 0) {
        const char* e = getenv("PE_GEMM_PDL");
        on = (e && e[0] == '0') ? 0 : 1;
    }
    return on;
}

// One persistent launch: clusters of `cluster` CTAs (1 = none), programmatic
// stream serialisation so that the prologue overlaps the previous kernel.
template <class C>
int launch_persistent(const GemmArgs& g, int grid, int cluster, cudaStream_t s) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(C::THREADS);
    cfg.dynamicSmemBytes = C::SMEM;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    int na = 0;
    if (cluster > 1) {
        attr[na].id = cudaLaunchAttributeClusterDimension;
        attr[na].val.clusterDim.x = cluster;
        attr[na].val.clusterDim.y = 1;
        attr[na].val.clusterDim.z = 1;
        ++na;
    }
    if (pdl_enabled()) {
        attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[na].val.programmaticStreamSerializationAllowed = 1;
        ++na;
    }
    cfg.attrs = attr;
    cfg.numAttrs = na;
    cudaError_t e = cudaLaunchKernelEx(&cfg, gemm_kernel<C>, g);
    count_launch();
    return check_cuda(e);
}

template <class C>
int launch_gemm(GemmArgs& g, cudaStream_t s) {
    // the shared-memory opt-in is a per-device function attribute
    static std::mutex mu;
    static bool done[64] = {false};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return set_last_error(PE_ERR_CUDA);
    {
        std::lock_guard<std::mutex> lk(mu);
        if (!done[dev]) {
            cudaError_t e = cudaFuncSetAttribute(gemm_kernel<C>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 C::SMEM);
            if (e != cudaSuccess) return check_cuda(e);
            done[dev] = true;
        }
    }
    g.mblk = (int)((g.M + C::TM - 1) / C::TM);
    g.nblk = (int)((g.N + C::BN - 1) / C::BN);
    g.kiters = (int)((g.K + C::BK - 1) / C::BK);
    if (g.sk_q > 0) {
        g.kper = g.kiters;  // unused: stream-K units come from sk_q
    } else if (g.ksplit <= 1 || g.kiters < 2) {
        g.ksplit = 1;
        g.kper = g.kiters;
    } else {
        g.kper = (g.kiters + g.ksplit - 1) / g.ksplit;
        g.ksplit = (g.kiters + g.kper - 1) / g.kper;  // every unit gets >= 1 k-iteration
    }
    int64_t tiles = (int64_t)g.mblk * g.nblk * (int64_t)g.tiles;  // g.tiles holds I on entry
    if (tiles > 0x7FFFFFFF) return set_last_error(PE_ERR_UNSUPPORTED);
    g.tiles = (int)tiles;
    if (g.sk_q > 0) {
        // the plan's slab count must cover every tile's segments
        if (C::PAIR || (g.kiters + g.sk_q - 1) / g.sk_q + 1 > g.ksplit) return set_last_error(PE_ERR_INVALID);
        const int64_t grid = (tiles * g.kiters + g.sk_q - 1) / g.sk_q;
        if (grid > num_sms()) return set_last_error(PE_ERR_INVALID);
        return launch_persistent<C>(g, (int)grid, 1, s);
    }
    if constexpr (C::PAIR) {
        // one cluster of two CTAs per tile pair, persistent over the SMs
        const int pairs = (int)std::min<int64_t>(tiles * g.ksplit, grid_cap() / 2);
        return launch_persistent<C>(g, 2 * pairs, 2, s);
    }
    const int grid = (int)std::min<int64_t>(tiles * g.ksplit, grid_cap());
    return launch_persistent<C>(g, grid, 1, s);
}

// fp32 3xTF32: the tensor core reads only the upper 19 bits of each fp32
// operand (sign, exponent, 10 mantissa bits) and ignores the low 13, so the
// TMA-landed x already acts as "big" and only "small" = x - big needs writing.
// PE_TF32_HW_TRUNC=0 restores the explicit masked write-back; a GPU test pins
// that both give bit-identical results.
// fp16 wide tiles run as CTA pairs (tcgen05 cta_group::2, 256x256 tiles)
// unless PE_GEMM_PAIRS=0.
// fp32 256-column tiles when both tf32 small halves are precomputed, unless
// PE_GEMM_WIDE_FP32=0.
int wide_fp32_enabled() {
    const char* e = getenv("PE_GEMM_WIDE_FP32");
    return (e && e[0] == '0') ? 0 : 1;
}

int thin_enabled() {
    const char* e = getenv("PE_THIN");
    return (e && e[0] == '0') ? 0 : 1;
}

int streamk_mode() {
    const char* e = getenv("PE_GEMM_STREAMK");
    if (e && e[0] == '0') return 0;
    if (e && e[0] == '2') return 2;
    return 1;
}

int pairs_enabled() {
    const char* e = getenv("PE_GEMM_PAIRS");
    return (e && e[0] == '0') ? 0 : 1;
}

// fp32 3xTF32 on CTA pairs (PE_GEMM_FP32_PAIRS=0 disables)
int fp32_pairs_enabled() {
    const char* e = getenv("PE_GEMM_FP32_PAIRS");
    return (e && e[0] == '0') ? 0 : 1;
}

// fp16 contraction rows per pipeline stage (1 or 2): PE_GEMM_KB overrides the
// default for CTA pairs and for single CTAs.
int stage_rows(bool pair) {
    const char* e = getenv("PE_GEMM_KB");
    if (e && (e[0] == '1' || e[0] == '2')) return e[0] - '0';
    return pair ? 2 : 1;
}

// fp32 fused-B MMAs on 128-column tiles (PE_GEMM_FUSEB=0 keeps three N=128 MMAs)
int fuse_b_enabled() {
    const char* e = getenv("PE_GEMM_FUSEB");
    return (e && e[0] == '0') ? 0 : 1;
}

// Epilogue warps of fp16 CTA pairs: 4 for long grids, else 8 (PE_EPI_WARPS_PAIR=4|8 forces)
int pair_epilogue_warps(bool long_grid) {
    const char* e = getenv("PE_EPI_WARPS_PAIR");
    if (e && e[0] == '4') return 4;
    if (e && e[0] == '8') return 8;
    return long_grid ? 4 : 8;
}

int raw_big_enabled() {
    const char* e = getenv("PE_TF32_HW_TRUNC");
    return (e && e[0] == '0') ? 0 : 1;
}

// Streaming contraction for degenerate shapes: one thread per output element
// (output order, so stores coalesce); products and sums in fp32 in the
// contraction order of the CPU reference, each rounded once, so fp32 results
// match it bit for bit.
struct SimtArgs {
    int nd, nk;
    FastDiv div[PE_MAX_RANK];                 // output axes (outermost first)
    int64_t sa[PE_MAX_RANK], sb[PE_MAX_RANK]; // their strides in A and B
    int64_t ksize[PE_MAX_RANK], ka[PE_MAX_RANK], kb[PE_MAX_RANK];  // contraction axes
    int64_t n, C;
};

// Four consecutive outputs along the innermost output axis per thread (its size
// a multiple of 4, output 16-byte aligned): one index decode and one 16-byte
// store per four elements; the same single-rounded products and sums as
// small_contract, so results are identical.
template <typename T>
__global__ void __launch_bounds__(256) small_contract4(const T* __restrict__ A, const T* __restrict__ B,
                                                       float* __restrict__ out, SimtArgs p) {
    const uint32_t n4 = (uint32_t)(p.n >> 2);
    const uint32_t step = gridDim.x * blockDim.x;
    const int64_t ia = p.sa[p.nd - 1], ib = p.sb[p.nd - 1];
    for (uint32_t e4 = blockIdx.x * blockDim.x + threadIdx.x; e4 < n4; e4 += step) {
        uint32_t rem = e4 << 2;
        int64_t ao = 0, bo = 0;
        for (int a = p.nd - 1; a >= 0; --a) {
            const uint32_t q = fdiv(rem, p.div[a]);
            const uint32_t idx = rem - q * p.div[a].div;
            rem = q;
            ao += (int64_t)idx * p.sa[a];
            bo += (int64_t)idx * p.sb[a];
        }
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        if (p.nk <= 1) {
            const int64_t ka = p.nk ? p.ka[0] : 0, kb = p.nk ? p.kb[0] : 0;
            for (int64_t c = 0; c < p.C; ++c) {
#pragma unroll
                for (int q = 0; q < 4; ++q)
                    acc[q] = __fadd_rn(acc[q], __fmul_rn((float)A[ao + q * ia + c * ka], (float)B[bo + q * ib + c * kb]));
            }
        } else {
            for (int64_t c = 0; c < p.C; ++c) {
                int64_t r = c, oa = ao, ob = bo;
                for (int a = p.nk - 1; a >= 0; --a) {
                    const int64_t q = r / p.ksize[a];
                    const int64_t idx = r - q * p.ksize[a];
                    r = q;
                    oa += idx * p.ka[a];
                    ob += idx * p.kb[a];
                }
#pragma unroll
                for (int q = 0; q < 4; ++q)
                    acc[q] = __fadd_rn(acc[q], __fmul_rn((float)A[oa + q * ia], (float)B[ob + q * ib]));
            }
        }
        *reinterpret_cast<float4*>(out + ((int64_t)e4 << 2)) = make_float4(acc[0], acc[1], acc[2], acc[3]);
    }
}

template <typename T>
__global__ void __launch_bounds__(256) small_contract(const T* __restrict__ A, const T* __restrict__ B,
                                                      float* __restrict__ out, SimtArgs p) {
    const uint32_t step = gridDim.x * blockDim.x;
    for (uint32_t e = blockIdx.x * blockDim.x + threadIdx.x; e < (uint32_t)p.n; e += step) {
        uint32_t rem = e;
        int64_t ao = 0, bo = 0;
        for (int a = p.nd - 1; a >= 0; --a) {
            const uint32_t q = fdiv(rem, p.div[a]);
            const uint32_t idx = rem - q * p.div[a].div;
            rem = q;
            ao += (int64_t)idx * p.sa[a];
            bo += (int64_t)idx * p.sb[a];
        }
        float acc = 0.f;
        if (p.nk <= 1) {
            const int64_t ka = p.nk ? p.ka[0] : 0, kb = p.nk ? p.kb[0] : 0;
            for (int64_t c = 0; c < p.C; ++c)
                acc = __fadd_rn(acc, __fmul_rn((float)A[ao + c * ka], (float)B[bo + c * kb]));
        } else {
            for (int64_t c = 0; c < p.C; ++c) {
                int64_t r = c, oa = ao, ob = bo;
                for (int a = p.nk - 1; a >= 0; --a) {
                    const int64_t q = r / p.ksize[a];
                    const int64_t idx = r - q * p.ksize[a];
                    r = q;
                    oa += idx * p.ka[a];
                    ob += idx * p.kb[a];
                }
                acc = __fadd_rn(acc, __fmul_rn((float)A[oa], (float)B[ob]));
            }
        }
        out[e] = acc;
    }
}

// Thin contraction: outputs with a free dimension of at most 4 whose
// contraction is one contiguous run in both operands (dot products,
// matrix-vector products, their batched forms). Work item = (output element,
// chunk of the contraction), one warp each: 16-byte loads of both operands,
// four fp32 accumulators per lane (fused multiply-add), then a fixed shuffle
// tree, so results are run-to-run identical. With several chunks the partial
// sums go to `part` ([chunk][output]) and a fixed-order reduction adds them.
struct ThinArgs {
    SimtArgs s;          // output decode; s.C = contraction length
    int64_t chunk;       // contraction elements per work item (multiple of 64)
    int nchunk;
    int aligned;         // both base pointers 16-byte aligned
};

template <typename T>
__device__ __forceinline__ void fma_vec(const uint4& x, const uint4& y, float& a0, float& a1) {
    if constexpr (sizeof(T) == 4) {
        a0 = fmaf(__uint_as_float(x.x), __uint_as_float(y.x), a0);
        a1 = fmaf(__uint_as_float(x.y), __uint_as_float(y.y), a1);
        a0 = fmaf(__uint_as_float(x.z), __uint_as_float(y.z), a0);
        a1 = fmaf(__uint_as_float(x.w), __uint_as_float(y.w), a1);
    } else {
        const __half2* hx = reinterpret_cast<const __half2*>(&x);
        const __half2* hy = reinterpret_cast<const __half2*>(&y);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const float2 fx = __half22float2(hx[q]), fy = __half22float2(hy[q]);
            a0 = fmaf(fx.x, fy.x, a0);
            a1 = fmaf(fx.y, fy.y, a1);
        }
    }
}

template <typename T>
__global__ void __launch_bounds__(256) thin_contract(const T* __restrict__ A, const T* __restrict__ B,
                                                     float* __restrict__ out, float* __restrict__ part,
                                                     ThinArgs p) {
    constexpr int VEC = 16 / sizeof(T);
    const int lane = threadIdx.x & 31;
    const int64_t nwork = p.s.n * p.nchunk;
    const int64_t wstep = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t w = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); w < nwork; w += wstep) {
        const int64_t e = w / p.nchunk;
        const int j = (int)(w - e * p.nchunk);
        uint32_t rem = (uint32_t)e;
        int64_t ao = 0, bo = 0;
        for (int a = p.s.nd - 1; a >= 0; --a) {
            const uint32_t q = fdiv(rem, p.s.div[a]);
            const uint32_t idx = rem - q * p.s.div[a].div;
            rem = q;
            ao += (int64_t)idx * p.s.sa[a];
            bo += (int64_t)idx * p.s.sb[a];
        }
        const int64_t c0 = (int64_t)j * p.chunk;
        const int64_t c1 = min(p.s.C, c0 + p.chunk);
        const T* a = A + ao;
        const T* b = B + bo;
        float acc0 = 0.f, acc1 = 0.f, acc2 = 0.f, acc3 = 0.f;
        int64_t c = c0;
        if (p.aligned && (ao % VEC) == 0 && (bo % VEC) == 0) {
            // two 16-byte vectors per operand and lane in flight per step
            for (; c + 64 * VEC <= c1; c += 64 * VEC) {
                const uint4 x0 = __ldcs(reinterpret_cast<const uint4*>(a + c + lane * VEC));
                const uint4 y0 = __ldcs(reinterpret_cast<const uint4*>(b + c + lane * VEC));
                const uint4 x1 = __ldcs(reinterpret_cast<const uint4*>(a + c + (32 + lane) * VEC));
                const uint4 y1 = __ldcs(reinterpret_cast<const uint4*>(b + c + (32 + lane) * VEC));
                fma_vec<T>(x0, y0, acc0, acc1);
                fma_vec<T>(x1, y1, acc2, acc3);
            }
        }
        for (c += lane; c < c1; c += 32) acc0 = fmaf((float)a[c], (float)b[c], acc0);
        float sum = (acc0 + acc1) + (acc2 + acc3);
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) sum += __shfl_down_sync(0xffffffffu, sum, off);
        if (lane == 0) {
            if (p.nchunk == 1) out[e] = sum;
            else part[(int64_t)j * p.s.n + e] = sum;
        }
    }
}

// Thin partials [chunk][output] -> out[output]: one warp per output, lanes
// take chunks j = lane, lane + 32, ... in order, then a fixed shuffle tree
// (run-to-run identical).
__global__ void __launch_bounds__(256) thin_reduce(const float* __restrict__ part, float* __restrict__ out,
                                                   int64_t n, int nchunk) {
    const int lane = threadIdx.x & 31;
    const int64_t wstep = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t e = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); e < n; e += wstep) {
        float acc = 0.f;
        for (int j = lane; j < nchunk; j += 32) acc += part[(int64_t)j * n + e];
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) acc += __shfl_down_sync(0xffffffffu, acc, off);
        if (lane == 0) out[e] = acc;
    }
}

// Many partials per output (dot products): a 256-thread block per output;
// thread k sums partials k, k + 256, ... with four accumulators in a fixed
// pattern, then a fixed shared-memory tree (run-to-run identical).
__global__ void __launch_bounds__(256) thin_reduce_block(const float* __restrict__ part, float* __restrict__ out,
                                                         int64_t n, int nchunk) {
    __shared__ float red[256];
    for (int64_t e = blockIdx.x; e < n; e += gridDim.x) {
        float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
        int j = threadIdx.x;
        for (; j + 768 < nchunk; j += 1024) {
            a0 += part[(int64_t)j * n + e];
            a1 += part[(int64_t)(j + 256) * n + e];
            a2 += part[(int64_t)(j + 512) * n + e];
            a3 += part[(int64_t)(j + 768) * n + e];
        }
        for (; j < nchunk; j += 256) a0 += part[(int64_t)j * n + e];
        red[threadIdx.x] = (a0 + a1) + (a2 + a3);
        __syncthreads();
        for (int w = 128; w > 0; w >>= 1) {
            if (threadIdx.x < w) red[threadIdx.x] += red[threadIdx.x + w];
            __syncthreads();
        }
        if (threadIdx.x == 0) out[e] = red[0];
        __syncthreads();
    }
}

template <typename T>
int thin_resident_blocks() {
    static int n = 0;
    if (n == 0) {
        int b = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, thin_contract<T>, 256, 0) != cudaSuccess || b <= 0)
            b = 4;
        n = b;
    }
    return n;
}

// tf32 "small" half of fp32 data: y = x - (x with its low 13 mantissa bits
// cleared). x - trunc(x) is exact in fp32. Up to two operands per launch
// (blockIdx.y selects the range).
struct SmallRange {
    const float* x;
    float* y;
    int64_t n;
};

__global__ void __launch_bounds__(256) tf32_small(SmallRange r0, SmallRange r1) {
    const SmallRange r = blockIdx.y ? r1 : r0;
    const float* __restrict__ x = r.x;
    float* __restrict__ y = r.y;
    const int64_t n = r.n;
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t step = (int64_t)gridDim.x * blockDim.x;
    const int64_t n4 = n / 4;
    for (int64_t v = i; v < n4; v += step) {
        const float4 a = reinterpret_cast<const float4*>(x)[v];
        float4 o;
        o.x = a.x - __uint_as_float(__float_as_uint(a.x) & 0xFFFFE000u);
        o.y = a.y - __uint_as_float(__float_as_uint(a.y) & 0xFFFFE000u);
        o.z = a.z - __uint_as_float(__float_as_uint(a.z) & 0xFFFFE000u);
        o.w = a.w - __uint_as_float(__float_as_uint(a.w) & 0xFFFFE000u);
        reinterpret_cast<float4*>(y)[v] = o;
    }
    for (int64_t e = 4 * n4 + i; e < n; e += step) y[e] = x[e] - __uint_as_float(__float_as_uint(x[e]) & 0xFFFFE000u);
}

// a.n or b.n may be 0 (operand not precomputed); nothing launches if both are.
int tf32_small_launch(SmallRange a, SmallRange b, cudaStream_t s) {
    if (a.n == 0) std::swap(a, b);
    if (a.n == 0) return PE_OK;
    const int ny = b.n ? 2 : 1;
    const int64_t nmax = std::max(a.n, b.n);
    int64_t blocks = (nmax / 4 + 255) / 256 + 1, cap = (int64_t)num_sms() * 8 / ny;
    tf32_small<<<dim3((unsigned)std::min(blocks, cap), ny), 256, 0, s>>>(a, b);
    count_launch();
    return check_cuda(cudaGetLastError());
}

// Split-K reduction: out[perm(e)] = sum over sp of part[sp][e] (fixed order,
// so results are run-to-run identical). e walks the canonical [I, L0, L1]
// index; `od` decodes it into the permuted output offset.
__global__ void __launch_bounds__(256) splitk_reduce(const float* __restrict__ part, float* __restrict__ out,
                                                     int64_t n, int ks, Decode od) {
    int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t step = (int64_t)gridDim.x * blockDim.x;
    for (; e < n; e += step) {
        float acc = part[e];
        for (int k = 1; k < ks; ++k) acc += part[(int64_t)k * n + e];
        out[decode_off(od, e)] = acc;
    }
}

// Stream-K reduction: element e of tile t sums the nseg(t) partial slabs of
// that tile's segments in slab order (fixed, so results are run-to-run
// identical); nseg follows from where the CTA boundaries (multiples of q in
// the flattened (tile, k) space) fall inside the tile.
struct SkReduce {
    int64_t L0, L1, per_batch, q;
    int nblk, tm, bn, kiters;
};

__global__ void __launch_bounds__(256) streamk_reduce(const float* __restrict__ part, float* __restrict__ out,
                                                      int64_t n, SkReduce r, Decode od) {
    int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t step = (int64_t)gridDim.x * blockDim.x;
    const int64_t plane = r.L0 * r.L1;
    for (; e < n; e += step) {
        const int64_t i = e / plane, rem = e - i * plane;
        const int64_t m = rem / r.L1, nn = rem - m * r.L1;
        const int64_t t = i * r.per_batch + (m / r.tm) * r.nblk + nn / r.bn;
        const int64_t base = t * r.kiters;
        const int ns = (int)((base + r.kiters - 1) / r.q - base / r.q + 1);
        float acc = part[e];
        for (int k = 1; k < ns; ++k) acc += part[(int64_t)k * n + e];
        out[decode_off(od, e)] = acc;
    }
}

struct Lowered;
int splitk_reduce_launch(const float* part, float* out, const Lowered& L, const pe_contract_plan* pl, int ks,
                         cudaStream_t s);

struct Lowered {
    OperandView a, b;
    bool a_ws = false, b_ws = false;
    int64_t kpad = 0;             // padded row length of workspace operands
    size_t a_off = 0, b_off = 0, p_off = 0, ws_bytes = 0;
    // fp32: precomputed tf32 "small" halves (same layout as the raw operand)
    bool a_pre = false, b_pre = false;
    size_t as_off = 0, bs_off = 0;
    int64_t n_in0 = 0, n_in1 = 0;        // raw operand element counts
    int bn = 128;                 // N tile of the chosen kernel
    bool simt = false;            // degenerate shape: streaming kernel instead of the GEMM
    bool thin = false;            // thin output, contiguous contraction: warp-per-dot kernel
    int64_t thin_chunk = 0, thin_nchunk = 1;
    int ksplit = 1;               // split-K factor (partials in the workspace when > 1)
    int64_t sk_q = 0;             // stream-K iterations per CTA (0 = off); ksplit = slab count then
    // group axes
    Axis a_batch[PE_MAX_RANK], a_free[PE_MAX_RANK], a_ct[PE_MAX_RANK];
    Axis b_batch[PE_MAX_RANK], b_free[PE_MAX_RANK], b_ct[PE_MAX_RANK];
    int nb = 0, n0 = 0, n1 = 0, nc = 0;
    OutView out;
};

// Contraction axes of the plan merged where they are contiguous in both
// operands (outermost first). Returns the number of merged axes.
int coalesce_contraction(const Lowered& L, int64_t* ksize, int64_t* ka, int64_t* kb) {
    int nk = 0;
    for (int j = 0; j < L.nc; ++j) {
        if (L.a_ct[j].size == 1) continue;
        if (nk > 0 && ka[nk - 1] == L.a_ct[j].stride * L.a_ct[j].size &&
            kb[nk - 1] == L.b_ct[j].stride * L.b_ct[j].size) {
            ksize[nk - 1] *= L.a_ct[j].size;
            ka[nk - 1] = L.a_ct[j].stride;
            kb[nk - 1] = L.b_ct[j].stride;
        } else {
            ksize[nk] = L.a_ct[j].size;
            ka[nk] = L.a_ct[j].stride;
            kb[nk] = L.b_ct[j].stride;
            nk++;
        }
    }
    return nk;
}

bool valid_perm(const int32_t* p, int n) {
    bool seen[PE_MAX_RANK] = {false};
    for (int a = 0; a < n; ++a) {
        if (p[a] < 0 || p[a] >= n || seen[p[a]]) return false;
        seen[p[a]] = true;
    }
    return true;
}

int lower(const pe_contract_plan* pl, const void* in0, const void* in1, Lowered* L) {
    if (!pl || (pl->dtype != PE_F32 && pl->dtype != PE_F16)) return PE_ERR_INVALID;
    const int nb = pl->n_batch, n0 = pl->n_free0, n1 = pl->n_free1, nc = pl->n_contract;
    if (nb < 0 || n0 < 0 || n1 < 0 || nc < 0) return PE_ERR_INVALID;
    if (pl->rank0 != nb + n0 + nc || pl->rank1 != nb + nc + n1 || pl->out_rank != nb + n0 + n1 ||
        pl->rank0 > PE_MAX_RANK || pl->rank1 > PE_MAX_RANK || pl->out_rank > PE_MAX_RANK)
        return PE_ERR_INVALID;
    if (!valid_perm(pl->perm0, pl->rank0) || !valid_perm(pl->perm1, pl->rank1) ||
        !valid_perm(pl->out_perm, pl->out_rank))
        return PE_ERR_INVALID;
    const int es = pl->dtype == PE_F32 ? 4 : 2;
    L->nb = nb;
    L->n0 = n0;
    L->n1 = n1;
    L->nc = nc;
    int64_t st0[PE_MAX_RANK], st1[PE_MAX_RANK], sto[PE_MAX_RANK], out_shape[PE_MAX_RANK];
    int64_t run = 1;
    for (int a = pl->rank0 - 1; a >= 0; --a) { st0[a] = run; run *= pl->shape0[a]; }
    run = 1;
    for (int a = pl->rank1 - 1; a >= 0; --a) { st1[a] = run; run *= pl->shape1[a]; }
    for (int p = 0; p < pl->out_rank; ++p) out_shape[p] = pl->out_interp_shape[pl->out_perm[p]];
    run = 1;
    int64_t interp_stride[PE_MAX_RANK];
    for (int p = pl->out_rank - 1; p >= 0; --p) { sto[p] = run; run *= out_shape[p]; }
    for (int p = 0; p < pl->out_rank; ++p) interp_stride[pl->out_perm[p]] = sto[p];
    // group axes (sizes from the raw shapes, consistency with I/L0/L1/C checked)
    int64_t I = 1, L0 = 1, L1 = 1, C = 1;
    for (int j = 0; j < nb; ++j) {
        int a0 = pl->perm0[j], a1 = pl->perm1[j];
        if (pl->shape0[a0] != pl->shape1[a1]) return PE_ERR_INVALID;
        L->a_batch[j] = {pl->shape0[a0], st0[a0]};
        L->b_batch[j] = {pl->shape1[a1], st1[a1]};
        L->out.b[j] = {pl->shape0[a0], interp_stride[j]};
        I *= pl->shape0[a0];
    }
    for (int j = 0; j < n0; ++j) {
        int a0 = pl->perm0[nb + j];
        L->a_free[j] = {pl->shape0[a0], st0[a0]};
        L->out.m[j] = {pl->shape0[a0], interp_stride[nb + j]};
        L0 *= pl->shape0[a0];
    }
    for (int j = 0; j < nc; ++j) {
        int a0 = pl->perm0[nb + n0 + j], a1 = pl->perm1[nb + j];
        if (pl->shape0[a0] != pl->shape1[a1]) return PE_ERR_INVALID;
        L->a_ct[j] = {pl->shape0[a0], st0[a0]};
        L->b_ct[j] = {pl->shape1[a1], st1[a1]};
        C *= pl->shape0[a0];
    }
    for (int j = 0; j < n1; ++j) {
        int a1 = pl->perm1[nb + nc + j];
        L->b_free[j] = {pl->shape1[a1], st1[a1]};
        L->out.n[j] = {pl->shape1[a1], interp_stride[nb + n0 + j]};
        L1 *= pl->shape1[a1];
    }
    L->out.nb = nb;
    L->out.nm = n0;
    L->out.nn = n1;
    if (I != pl->I || L0 != pl->L0 || L1 != pl->L1 || C != pl->C) return PE_ERR_INVALID;
    if (L0 > 0x7FFFFFFFll || L1 > 0x7FFFFFFFll || C > 0x7FFFFFFFll || I > 0xFFFFFFFFll)
        return PE_ERR_UNSUPPORTED;
    L->a = view_direct(in0, es, L->a_batch, nb, L->a_free, n0, L->a_ct, nc);
    L->b = view_direct(in1, es, L->b_batch, nb, L->b_free, n1, L->b_ct, nc);
    // validate tensor maps now so a rejected layout falls back to the workspace
    if (L->a.direct && in0) {
        CUtensorMap t;
        if (!encode_operand(&t, L->a, es == 4, 128)) L->a.direct = false;
    }
    if (L->b.direct && in1) {
        CUtensorMap t;
        if (!encode_operand(&t, L->b, es == 4, 128)) L->b.direct = false;
    }
    L->a_ws = !L->a.direct;
    L->b_ws = !L->b.direct;
    const int64_t vec = 16 / es;
    L->kpad = ((C > 0 ? C : 1) + vec - 1) / vec * vec;
    // Degenerate contractions (a free dim of at most 4 with a short
    // contraction, e.g. a broadcast planned as 262144 batches of 4x1x1) would
    // fill a 128-row MMA tile with almost nothing; they run on the streaming
    // kernel and need no scratch.
    // Contractions of at most 4 elements (outer products and the like) are a
    // pure output stream; the MMA path would pad K to a full k-step.
    L->simt = (std::min(L0, L1) <= 4 && C <= 64) || C <= 4;
    if (L->simt) {
        L->a_ws = L->b_ws = false;
        L->ws_bytes = 0;
        return PE_OK;
    }
    // Thin outputs over a long contraction that is one contiguous run in both
    // operands (dot products, matrix-vector products): an MMA tile would
    // compute up to 128x128 products per useful one, so a streaming kernel
    // with one warp per (output, contraction chunk) reads both operands once.
    if (std::min(L0, L1) <= 4 && C >= 256 && thin_enabled()) {
        int64_t ks[PE_MAX_RANK], ka[PE_MAX_RANK], kb[PE_MAX_RANK];
        const int nk = coalesce_contraction(*L, ks, ka, kb);
        const int64_t n_out = I * L0 * L1;
        if (nk == 1 && ka[0] == 1 && kb[0] == 1 && n_out < (1ll << 31)) {
            const int64_t want = (int64_t)num_sms() * 64 * 4;  // four work items per resident warp
            int64_t nch = std::max<int64_t>(1, std::min<int64_t>((want + n_out - 1) / n_out, C / 1024));
            int64_t chunk = ((C + nch - 1) / nch + 63) / 64 * 64;
            nch = (C + chunk - 1) / chunk;
            L->thin = true;
            L->thin_chunk = chunk;
            L->thin_nchunk = nch;
            L->a_ws = L->b_ws = false;
            L->p_off = 0;
            L->ws_bytes = nch > 1 ? (((size_t)nch * n_out * 4 + 255) & ~(size_t)255) : 0;
            return PE_OK;
        }
    }
    size_t off = 0;
    if (L->a_ws) {
        L->a_off = off;
        off += ((size_t)I * L0 * L->kpad * es + 255) & ~(size_t)255;
    }
    if (L->b_ws) {
        L->b_off = off;
        off += ((size_t)I * L1 * L->kpad * es + 255) & ~(size_t)255;
    }
    // Tile shape and split-K. Thin outputs with long contractions leave SMs
    // idle; splitting K into `ks` ranges fills them at the price of writing and
    // re-reading ks fp32 partial slabs. Pick ks minimising
    // (waves of units / ks) + (partial traffic / input traffic).
    const int nsm = num_sms();
    const int64_t mblk = (L0 + 127) / 128;
    if (es == 2) {
        const int64_t tiles256 = I * mblk * ((L1 + 255) / 256);
        L->bn = (L1 > 128 && tiles256 >= nsm) ? 256 : 128;
    }
    const int64_t tiles = I * mblk * ((L1 + L->bn - 1) / L->bn);
    const int64_t kiters = (C + (128 / es) - 1) / (128 / es);
    const double in_bytes = (double)es * (double)C * (double)(I * L0 + I * L1);
    const double part_bytes = 8.0 * (double)(I * L0 * L1);
    double best = 1.0;
    if (tiles > 0 && tiles * 2 <= nsm && kiters >= 64) {
        for (int ks = 2; ks <= 16 && ks <= kiters / 8; ++ks) {
            const double waves = (double)((tiles * ks + nsm - 1) / nsm) / ks;
            const double cost = waves + ks * part_bytes / in_bytes;
            if (cost < best - 0.02) {
                best = cost;
                L->ksplit = ks;
            }
        }
    }
    // Stream-K: every CTA takes an equal share of the flattened (tile, k)
    // iterations, so all SMs stay busy whatever the tile count; a tile touched
    // by several CTAs gets one partial per CTA boundary inside it.
    // PE_GEMM_STREAMK=0 disables it, =2 forces it wherever it can apply.
    const int skm = streamk_mode();
    if (skm && tiles > 0 && tiles < nsm && kiters >= (skm == 2 ? 2 : 16)) {
        const int64_t total = tiles * kiters;
        const int64_t ncta = std::min<int64_t>(nsm, total / (skm == 2 ? 2 : 8));
        if (ncta > tiles) {
            const int64_t q = (total + ncta - 1) / ncta;
            const double segs = (double)(tiles + ncta - 1) / (double)tiles;
            // partial slabs that stay in L2 (small problems) cost far less than
            // their HBM bytes suggest
            const double l2_scale = (in_bytes + segs * part_bytes) < 48.0 * (1 << 20) ? 0.2 : 1.0;
            const double cost = (double)q / (double)kiters + l2_scale * segs * part_bytes / in_bytes;
            if (skm == 2 || cost < best - 0.02) {
                best = cost;
                L->sk_q = q;
                L->ksplit = (int)((kiters + q - 1) / q + 1);
            }
        }
    }
    // fp32 operands that are small next to the output get their tf32 small
    // halves computed once by a streaming pass instead of by the split warps
    // for every tile that reads them (4a: 4 MB operands, 268 MB output). An
    // operand read by a single tile along the other free dimension gains
    // nothing from the pass (it would only add a launch and a write + read of
    // the halves), so it keeps the in-kernel split.
    if (es == 4) {
        int64_t n0e = 1, n1e = 1;
        for (int a = 0; a < pl->rank0; ++a) n0e *= pl->shape0[a];
        for (int a = 0; a < pl->rank1; ++a) n1e *= pl->shape1[a];
        L->n_in0 = n0e;
        L->n_in1 = n1e;
        const int64_t cap = (int64_t)16 << 20;  // elements (64 MB)
        if (L->a.direct && n0e <= cap && L1 > 128) {
            L->a_pre = true;
            L->as_off = off;
            off += ((size_t)n0e * 4 + 255) & ~(size_t)255;
        }
        if (L->b.direct && n1e <= cap && L0 > 128) {
            L->b_pre = true;
            L->bs_off = off;
            off += ((size_t)n1e * 4 + 255) & ~(size_t)255;
        }
    }
    if (L->ksplit > 1) {
        L->p_off = off;
        off += ((size_t)L->ksplit * I * L0 * L1 * 4 + 255) & ~(size_t)255;
    }
    L->ws_bytes = off;
    return PE_OK;
}

// Gather one operand into the canonical [I, L, Kpad] K-major workspace.
int gather_canonical(int es, const void* src, void* dst, const Axis* batch, int nb, const Axis* fr,
                     int nf, const Axis* ct, int nc, int64_t L, int64_t kpad, cudaStream_t s) {
    int64_t size[PE_MAX_RANK], sst[PE_MAX_RANK], dst_st[PE_MAX_RANK];
    int nd = 0;
    // destination strides: contract axes contiguous, free axes x kpad, batch x L*kpad
    int64_t run = 1;
    int64_t dst_ct[PE_MAX_RANK], dst_fr[PE_MAX_RANK], dst_b[PE_MAX_RANK];
    for (int j = nc - 1; j >= 0; --j) { dst_ct[j] = run; run *= ct[j].size; }
    run = kpad;
    for (int j = nf - 1; j >= 0; --j) { dst_fr[j] = run; run *= fr[j].size; }
    run = L * kpad;
    for (int j = nb - 1; j >= 0; --j) { dst_b[j] = run; run *= batch[j].size; }
    for (int j = 0; j < nb; ++j) { size[nd] = batch[j].size; sst[nd] = batch[j].stride; dst_st[nd++] = dst_b[j]; }
    for (int j = 0; j < nf; ++j) { size[nd] = fr[j].size; sst[nd] = fr[j].stride; dst_st[nd++] = dst_fr[j]; }
    for (int j = 0; j < nc; ++j) { size[nd] = ct[j].size; sst[nd] = ct[j].stride; dst_st[nd++] = dst_ct[j]; }
    return strided_copy_launch(es, nd, size, sst, dst_st, src, dst, s);
}

int splitk_reduce_launch(const float* part, float* out, const Lowered& L, const pe_contract_plan* pl, int ks,
                         cudaStream_t s) {
    Axis ax[3 * PE_MAX_RANK];
    int n = 0;
    for (int j = 0; j < L.out.nb; ++j) ax[n++] = L.out.b[j];
    for (int j = 0; j < L.out.nm; ++j) ax[n++] = L.out.m[j];
    for (int j = 0; j < L.out.nn; ++j) ax[n++] = L.out.n[j];
    Axis c[3 * PE_MAX_RANK];
    int k = coalesce(ax, n, c);
    if (k > PE_MAX_RANK) return set_last_error(PE_ERR_UNSUPPORTED);
    Decode od = make_decode(c, k);
    const int64_t total = pl->I * pl->L0 * pl->L1;
    int64_t blocks = (total + 255) / 256, cap = (int64_t)num_sms() * 8;
    splitk_reduce<<<(int)std::min(blocks, cap), 256, 0, s>>>(part, out, total, ks, od);
    count_launch();
    return check_cuda(cudaGetLastError());
}

int streamk_reduce_launch(const float* part, float* out, const Lowered& L, const pe_contract_plan* pl,
                          const GemmArgs& g, cudaStream_t s) {
    Axis ax[3 * PE_MAX_RANK];
    int n = 0;
    for (int j = 0; j < L.out.nb; ++j) ax[n++] = L.out.b[j];
    for (int j = 0; j < L.out.nm; ++j) ax[n++] = L.out.m[j];
    for (int j = 0; j < L.out.nn; ++j) ax[n++] = L.out.n[j];
    Axis c[3 * PE_MAX_RANK];
    int k = coalesce(ax, n, c);
    if (k > PE_MAX_RANK) return set_last_error(PE_ERR_UNSUPPORTED);
    Decode od = make_decode(c, k);
    SkReduce r;
    r.L0 = pl->L0;
    r.L1 = pl->L1;
    r.tm = 128;  // stream-K runs only on single-CTA 128-row tiles
    r.bn = L.bn;
    r.nblk = (int)((pl->L1 + r.bn - 1) / r.bn);
    r.per_batch = ((pl->L0 + r.tm - 1) / r.tm) * (int64_t)r.nblk;
    r.q = g.sk_q;
    r.kiters = g.kiters;
    const int64_t total = pl->I * pl->L0 * pl->L1;
    int64_t blocks = (total + 255) / 256, cap = (int64_t)num_sms() * 8;
    streamk_reduce<<<(int)std::min(blocks, cap), 256, 0, s>>>(part, out, total, r, od);
    count_launch();
    return check_cuda(cudaGetLastError());
}

// Output axes in output memory order with their A / B strides, and the
// merged contraction axes: the shared setup of the streaming kernels.
int build_simt_args(const pe_contract_plan* pl, const Lowered& L, SimtArgs& p) {
    p = SimtArgs{};
    const int nb = L.nb, n0 = L.n0, n1 = L.n1;
    // interp axis j -> (A stride, B stride)
    int64_t ia[PE_MAX_RANK], ib[PE_MAX_RANK], isz[PE_MAX_RANK];
    for (int j = 0; j < nb; ++j) { ia[j] = L.a_batch[j].stride; ib[j] = L.b_batch[j].stride; isz[j] = L.a_batch[j].size; }
    for (int j = 0; j < n0; ++j) { ia[nb + j] = L.a_free[j].stride; ib[nb + j] = 0; isz[nb + j] = L.a_free[j].size; }
    for (int j = 0; j < n1; ++j) { ia[nb + n0 + j] = 0; ib[nb + n0 + j] = L.b_free[j].stride; isz[nb + n0 + j] = L.b_free[j].size; }
    int64_t n = 1;
    for (int q = 0; q < pl->out_rank; ++q) {
        const int j = pl->out_perm[q];
        if (isz[j] == 1) continue;
        p.div[p.nd] = make_fastdiv((uint32_t)isz[j]);
        p.sa[p.nd] = ia[j];
        p.sb[p.nd] = ib[j];
        p.nd++;
        n *= isz[j];
    }
    p.nk = coalesce_contraction(L, p.ksize, p.ka, p.kb);
    p.n = n;
    p.C = pl->C;
    // 32-bit element indices and grid strides in the streaming kernels
    if (n >= (1ll << 31)) return set_last_error(PE_ERR_UNSUPPORTED);
    return PE_OK;
}

int small_contract_launch(const pe_contract_plan* pl, const Lowered& L, const void* in0, const void* in1,
                          float* out, cudaStream_t s) {
    SimtArgs p;
    if (int rc = build_simt_args(pl, L, p)) return rc;
    const int64_t n = p.n;
    // four outputs per thread where the innermost output axis allows it
    if (p.nd >= 1 && p.div[p.nd - 1].div % 4 == 0 && ((uintptr_t)out & 15) == 0) {
        const int grid4 = (int)((n / 4 + 255) / 256);
        if (pl->dtype == PE_F32)
            small_contract4<float><<<grid4, 256, 0, s>>>((const float*)in0, (const float*)in1, out, p);
        else
            small_contract4<__half><<<grid4, 256, 0, s>>>((const __half*)in0, (const __half*)in1, out, p);
        count_launch();
        return check_cuda(cudaGetLastError());
    }
    // one output element per thread (n < 2^31): every element's operand loads
    // are in flight at once instead of a latency-bound walk per thread
    const int grid = (int)((n + 255) / 256);
    if (pl->dtype == PE_F32)
        small_contract<float><<<grid, 256, 0, s>>>((const float*)in0, (const float*)in1, out, p);
    else
        small_contract<__half><<<grid, 256, 0, s>>>((const __half*)in0, (const __half*)in1, out, p);
    count_launch();
    return check_cuda(cudaGetLastError());
}

int thin_contract_launch(const pe_contract_plan* pl, const Lowered& L, const void* in0, const void* in1,
                         float* out, void* ws, cudaStream_t s) {
    ThinArgs p;
    if (int rc = build_simt_args(pl, L, p.s)) return rc;
    if (p.s.nk != 1) return set_last_error(PE_ERR_INVALID);
    p.chunk = L.thin_chunk;
    p.nchunk = (int)L.thin_nchunk;
    p.aligned = ((uintptr_t)in0 % 16 == 0) && ((uintptr_t)in1 % 16 == 0);
    float* part = p.nchunk > 1 ? (float*)((uint8_t*)ws + L.p_off) : nullptr;
    if (p.nchunk > 1 && !ws) return set_last_error(PE_ERR_WORKSPACE);
    const int64_t warps = p.s.n * p.nchunk;
    const int res = pl->dtype == PE_F32 ? thin_resident_blocks<float>() : thin_resident_blocks<__half>();
    int64_t blocks = (warps + 7) / 8, cap = (int64_t)num_sms() * res;
    const int grid = (int)std::min(blocks, cap);
    if (pl->dtype == PE_F32)
        thin_contract<float><<<grid, 256, 0, s>>>((const float*)in0, (const float*)in1, out, part, p);
    else
        thin_contract<__half><<<grid, 256, 0, s>>>((const __half*)in0, (const __half*)in1, out, part, p);
    count_launch();
    int rc = check_cuda(cudaGetLastError());
    if (rc || p.nchunk == 1) return rc;
    // partials are in output memory order
    if (p.nchunk >= 1024) {
        thin_reduce_block<<<(int)std::min(p.s.n, (int64_t)num_sms() * 8), 256, 0, s>>>(part, out, p.s.n,
                                                                                      p.nchunk);
    } else {
        int64_t rb = (p.s.n + 7) / 8;
        thin_reduce<<<(int)std::min(rb, (int64_t)num_sms() * 8), 256, 0, s>>>(part, out, p.s.n, p.nchunk);
    }
    count_launch();
    return check_cuda(cudaGetLastError());
}

OperandView canonical_view(const void* base, int64_t I, int64_t L, int64_t C, int64_t kpad) {
    OperandView v;
    v.direct = true;
    v.mn_major = false;
    v.base = base;
    v.mn_size = L;
    v.mn_stride = kpad;
    v.k_size = C;
    v.k_stride = 1;
    v.nb = I > 1 ? 1 : 0;
    v.b_size[0] = I;
    v.b_stride[0] = L * kpad;
    return v;
}

// The launches of one contraction, prepared on the host (plan lowered, tensor
// maps encoded) and replayable: each step enqueues one kernel on the stream.
using Step = std::function<int(cudaStream_t)>;
using Program = std::vector<Step>;

int build_program(const pe_contract_plan& pl, const Lowered& L, const void* in0, const void* in1,
                  float* out, void* ws, int phase, Program& prog);

int run_program(const Program& prog, cudaStream_t s) {
    for (const Step& st : prog)
        if (int rc = st(s)) return rc;
    return set_last_error(PE_OK);
}

}  // namespace

int contract_workspace_bytes(const pe_contract_plan* plan, size_t* bytes) {
    if (!bytes) return set_last_error(PE_ERR_INVALID);
    Lowered L;
    // Without pointers the direct/workspace decision cannot see the base
    // alignment; use 16-byte aligned placeholders (torch allocations are).
    int rc = lower(plan, (const void*)256, (const void*)256, &L);
    if (rc) return set_last_error(rc);
    *bytes = L.ws_bytes;
    return set_last_error(PE_OK);
}

int contract_scratch_bytes(const pe_contract_plan* plan, const void* in0, const void* in1, size_t* bytes) {
    if (!bytes) return set_last_error(PE_ERR_INVALID);
    Lowered L;
    int rc = lower(plan, in0, in1, &L);
    if (rc) return set_last_error(rc);
    *bytes = L.ws_bytes;
    return set_last_error(PE_OK);
}

namespace {

// Lower the plan for these pointers and build its launch program. `tmp_bytes`
// > 0 means the caller's workspace is too small for this call (a misaligned
// view needs a gather the plan-time size did not include).
int prepare(const pe_contract_plan* pl, const void* in0, const void* in1, float* out, void* ws,
            size_t ws_bytes, int phase, Program& prog, size_t* tmp_bytes) {
    *tmp_bytes = 0;
    Lowered L;
    int rc = lower(pl, in0, in1, &L);
    if (rc) return set_last_error(rc);
    const int64_t n_out = pl->I * pl->L0 * pl->L1;
    if (n_out == 0) return set_last_error(PE_OK);
    if (!out) return set_last_error(PE_ERR_INVALID);
    if (pl->C == 0) {
        const size_t nb = (size_t)n_out * 4;
        if (phase < 3) return set_last_error(PE_OK);
        prog.push_back([out, nb](cudaStream_t s) { return check_cuda(cudaMemsetAsync(out, 0, nb, s)); });
        return set_last_error(PE_OK);
    }
    if (!in0 || !in1) return set_last_error(PE_ERR_INVALID);
    if (!L.simt && !get_encode()) return set_last_error(PE_ERR_NO_DEVICE);
    if (L.ws_bytes > 0 && (!ws || ws_bytes < L.ws_bytes)) {
        *tmp_bytes = L.ws_bytes;
        return set_last_error(PE_OK);
    }
    return build_program(*pl, L, in0, in1, out, ws, phase, prog);
}

// Per-workspace-handle cache of prepared programs, keyed by the exact
// pointers of the call: a repeat call replays its launches without lowering
// the plan or encoding tensor maps again.
struct CacheEntry {
    const pe_contract_plan* plan = nullptr;
    pe_contract_plan plan_copy;
    int phase = 3;
    const void* in0 = nullptr;
    const void* in1 = nullptr;
    float* out = nullptr;
    void* ws = nullptr;
    size_t ws_bytes = 0;
    uint64_t used = 0;
    Program prog;
};

struct ProgramCache {
    static constexpr int kEntries = 8;
    std::mutex mu;
    CacheEntry e[kEntries];
    uint64_t clock = 0;
};

}  // namespace

int contract_phase(const pe_contract_plan* pl, const void* in0, const void* in1, float* out, void* ws,
                   size_t ws_bytes, int phase, cudaStream_t s) {
    Program prog;
    size_t tmp_bytes = 0;
    int rc = prepare(pl, in0, in1, out, ws, ws_bytes, phase, prog, &tmp_bytes);
    if (rc) return rc;
    if (tmp_bytes == 0) return run_program(prog, s);
    // stream-ordered scratch for this call only
    void* tmp_ws = nullptr;
    rc = check_cuda(cudaMallocAsync(&tmp_ws, tmp_bytes, s));
    if (rc) return rc;
    rc = prepare(pl, in0, in1, out, tmp_ws, tmp_bytes, phase, prog, &tmp_bytes);
    if (!rc) rc = run_program(prog, s);
    int rc2 = check_cuda(cudaFreeAsync(tmp_ws, s));
    return rc ? rc : rc2;
}

int contract(const pe_contract_plan* pl, const void* in0, const void* in1, float* out, void* ws,
             size_t ws_bytes, cudaStream_t s) {
    return contract_phase(pl, in0, in1, out, ws, ws_bytes, 3, s);
}

void* program_cache_create() { return new ProgramCache(); }

void program_cache_destroy(void* c) { delete (ProgramCache*)c; }

int contract_cached(void* cache, const pe_contract_plan* pl, const void* in0, const void* in1, float* out,
                    void* ws, size_t ws_bytes, int phase, cudaStream_t s) {
    ProgramCache* pc = (ProgramCache*)cache;
    // PE_PLAN_CACHE=0 turns the cache off (every call lowers and encodes again)
    static const bool enabled = [] {
        const char* e = getenv("PE_PLAN_CACHE");
        return !(e && e[0] == '0');
    }();
    if (!pc || !pl || !enabled) return contract_phase(pl, in0, in1, out, ws, ws_bytes, phase, s);
    std::lock_guard<std::mutex> lk(pc->mu);
    CacheEntry* victim = &pc->e[0];
    for (CacheEntry& e : pc->e) {
        if (e.plan == pl && e.phase == phase && e.in0 == in0 && e.in1 == in1 && e.out == out && e.ws == ws &&
            e.ws_bytes == ws_bytes && memcmp(&e.plan_copy, pl, sizeof(*pl)) == 0) {
            e.used = ++pc->clock;
            return run_program(e.prog, s);
        }
        if (e.used < victim->used) victim = &e;
    }
    Program prog;
    size_t tmp_bytes = 0;
    int rc = prepare(pl, in0, in1, out, ws, ws_bytes, phase, prog, &tmp_bytes);
    if (rc) return rc;
    if (tmp_bytes) return contract_phase(pl, in0, in1, out, ws, ws_bytes, phase, s);  // not cached
    rc = run_program(prog, s);
    if (rc) return rc;
    victim->plan = pl;
    victim->plan_copy = *pl;
    victim->phase = phase;
    victim->in0 = in0;
    victim->in1 = in1;
    victim->out = out;
    victim->ws = ws;
    victim->ws_bytes = ws_bytes;
    victim->used = ++pc->clock;
    victim->prog = std::move(prog);
    return rc;
}

namespace {
int build_program(const pe_contract_plan& plan, const Lowered& L, const void* in0, const void* in1,
                  float* out, void* ws, int phase, Program& prog) {
    const pe_contract_plan* pl = &plan;
    // phase gate (EINSUM_PHASE_STOP): the single-phase streaming kernels run only
    // in full builds; the fused GEMM keeps its barrier skeleton at every level
    if ((L.simt || L.thin) && phase < 3) return set_last_error(PE_OK);
    if (L.simt) {
        prog.push_back([plan, L, in0, in1, out](cudaStream_t s) {
            return small_contract_launch(&plan, L, in0, in1, out, s);
        });
        return set_last_error(PE_OK);
    }
    if (L.thin) {
        prog.push_back([plan, L, in0, in1, out, ws](cudaStream_t s) {
            return thin_contract_launch(&plan, L, in0, in1, out, ws, s);
        });
        return set_last_error(PE_OK);
    }
    const int es = pl->dtype == PE_F32 ? 4 : 2;
    OperandView va = L.a, vb = L.b;
    if (L.a_ws) {
        void* dst = (uint8_t*)ws + L.a_off;
        const int64_t L0 = pl->L0, kpad = L.kpad;
        if (phase >= 1) prog.push_back([es, in0, dst, L, L0, kpad](cudaStream_t s) {
            return gather_canonical(es, in0, dst, L.a_batch, L.nb, L.a_free, L.n0, L.a_ct, L.nc, L0, kpad, s);
        });
        va = canonical_view(dst, pl->I, pl->L0, pl->C, L.kpad);
    }
    if (L.b_ws) {
        void* dst = (uint8_t*)ws + L.b_off;
        const int64_t L1 = pl->L1, kpad = L.kpad;
        if (phase >= 1) prog.push_back([es, in1, dst, L, L1, kpad](cudaStream_t s) {
            return gather_canonical(es, in1, dst, L.b_batch, L.nb, L.b_free, L.n1, L.b_ct, L.nc, L1, kpad, s);
        });
        vb = canonical_view(dst, pl->I, pl->L1, pl->C, L.kpad);
    }
    GemmArgs g;
    memset(&g, 0, sizeof(g));
    g.M = (int)pl->L0;
    g.N = (int)pl->L1;
    g.K = (int)pl->C;
    g.a_mn = va.mn_major;
    g.b_mn = vb.mn_major;
    g.ab = map_batch(va);
    g.bb = map_batch(vb);
    g.ksplit = L.ksplit;
    g.sk_q = (int)L.sk_q;
    g.nbatch = (int)pl->I;
    g.raw_big = raw_big_enabled();
    g.phase = phase;
    OutView slab;  // split-K: canonical partial slabs [ksplit * I, L0, L1]
    const OutView* ov = &L.out;
    float* target = out;
    if (L.ksplit > 1) {
        slab.nb = slab.nm = slab.nn = 1;
        slab.b[0] = {(int64_t)L.ksplit * pl->I, pl->L0 * pl->L1};
        slab.m[0] = {pl->L0, pl->L1};
        slab.n[0] = {pl->L1, 1};
        ov = &slab;
        target = (float*)((uint8_t*)ws + L.p_off);
    }
    g.out = target;
    {
        // the layout check of a tensor map over the output: unit-stride rows with
        // 16-byte aligned strides, at most three batch axes
        CUtensorMap tm_check;
        MapBatch mb_check;
        g.out_rows = encode_output(&tm_check, target, *ov, &mb_check) ? 1 : 0;
        g.out_v8 = g.out_rows && rows_aligned32(target, *ov) ? 1 : 0;  // narrowed per variant below
    }
    g.ob = make_decode(ov->b, ov->nb);
    g.om = make_decode(ov->m, ov->nm);
    g.on = make_decode(ov->n, ov->nn);
    g.tiles = (int)pl->I;
    // the GEMM step launches a copy: launch_gemm fills in the tile counts
    auto gemm_step = [&prog](auto cfg_tag, const GemmArgs& ga) {
        using C = decltype(cfg_tag);
        prog.push_back([ga](cudaStream_t s) {
            GemmArgs gg = ga;
            return launch_gemm<C>(gg, s);
        });
    };
    const bool f32 = pl->dtype == PE_F32;
    if (f32) {
        // more slots for long contractions: fewer accumulation steps per slot
        const int64_t kit = (pl->C + 31) / 32;
        g.acc_slots = kit >= 32 ? 4 : (kit >= 8 ? 2 : 1);
        SmallRange ra{nullptr, nullptr, 0}, rb{nullptr, nullptr, 0};
        if (L.a_pre) {
            void* sm = (uint8_t*)ws + L.as_off;
            ra = SmallRange{(const float*)in0, (float*)sm, L.n_in0};
            OperandView v = va;
            v.base = sm;
            if (!encode_operand(&g.tmas, v, true, 128)) return set_last_error(PE_ERR_UNSUPPORTED);
            g.a_pre = 1;
        }
        if (L.b_pre) {
            void* sm = (uint8_t*)ws + L.bs_off;
            rb = SmallRange{(const float*)in1, (float*)sm, L.n_in1};
            OperandView v = vb;
            v.base = sm;
            if (!encode_operand(&g.tmbs, v, true, 128)) return set_last_error(PE_ERR_UNSUPPORTED);
            g.b_pre = 1;
        }
        if ((ra.n || rb.n) && phase >= 1) prog.push_back([ra, rb](cudaStream_t s) { return tf32_small_launch(ra, rb, s); });
        if (!encode_operand(&g.tma, va, true, 128) || !encode_operand(&g.tmb, vb, true, 128))
            return set_last_error(PE_ERR_UNSUPPORTED);
        // both small halves precomputed: the split warps have nothing to do, so
        // spend the threads on epilogue warps instead (output-bound shapes)
        const int64_t tiles256 = pl->I * ((pl->L0 + 127) / 128) * ((pl->L1 + 255) / 256);
        const int64_t tiles256x2 = pl->I * ((pl->L0 + 255) / 256) * ((pl->L1 + 255) / 256);
        if (g.a_pre && g.b_pre && pl->L1 >= 256 && g.acc_slots <= 2 && tiles256x2 >= num_sms() / 2 &&
            L.sk_q == 0 && L.ksplit <= 1 && wide_fp32_enabled() && pairs_enabled() && fp32_pairs_enabled()) {
            // CTA pairs on 256x256 tiles: each SM lands its 128 rows of A and half
            // of B (raw and small halves), so per-SM operand traffic falls by a
            // quarter on this shared-memory-bound path
            OperandView vbs = vb;
            vbs.base = (uint8_t*)ws + L.bs_off;
            if (!encode_operand(&g.tmb, vb, true, 128) || !encode_operand(&g.tmbs, vbs, true, 128))
                return set_last_error(PE_ERR_UNSUPPORTED);
            g.out_v8 &= epi_v8_enabled(false);
            gemm_step(Cfg<256, true, 8, true, 0>{}, g);
        } else if (g.a_pre && g.b_pre && pl->L1 >= 256 && g.acc_slots <= 2 && tiles256 >= num_sms() &&
            wide_fp32_enabled()) {
            // wide tiles halve the tf32 MMA count per output column block
            OperandView vbs = vb;
            vbs.base = (uint8_t*)ws + L.bs_off;
            if (!encode_operand(&g.tmb, vb, true, 256) || !encode_operand(&g.tmbs, vbs, true, 256))
                return set_last_error(PE_ERR_UNSUPPORTED);
            g.out_v8 &= epi_v8_enabled(false);
            gemm_step(Cfg<256, true, 8, false, 0>{}, g);
        } else {
            // 128-column tiles: fused-B MMAs from two k-steps on (both rotation slots used)
            if (g.acc_slots >= 2 && fuse_b_enabled()) {
                g.fuse_b = 1;
                g.acc_slots = 4;
            }
            g.out_v8 &= epi_v8_enabled(false);
            if (g.a_pre && g.b_pre)
                gemm_step(Cfg<128, true, 8, false, 0>{}, g);
            else
                gemm_step(Cfg<128, true>{}, g);
        }
    } else {
        // pairs halve each SM's operand traffic, which pays off where the
        // mainloop dominates (long K); output-bound short-K shapes stay single
        const bool pair = L.bn == 256 && g.K >= 512 && L.sk_q == 0 && pairs_enabled();
        // two 128-byte contraction rows per stage (unsplit launches only: the
        // split-K reductions count k-iterations of one row)
        const int kb = (L.ksplit <= 1 && L.sk_q == 0) ? stage_rows(pair) : 1;
        const int box_k = kb == 2 ? 128 : 0;
        if (!encode_operand(&g.tma, va, false, 128, box_k) ||
            !encode_operand(&g.tmb, vb, false, pair ? 128 : L.bn, box_k))
            return set_last_error(PE_ERR_UNSUPPORTED);
        g.out_v8 &= epi_v8_enabled(pair);
        // four epilogue warps once there are four or more waves of pair tiles: the
        // stores spread over the mainloop they hide under (config 2: 144.3 -> 142.3 us);
        // short grids keep eight, whose last tile's stores have nothing to hide under
        const int64_t pair_tiles = pl->I * ((pl->L0 + 255) / 256) * ((pl->L1 + 255) / 256);
        if (pair && kb == 2 && pair_epilogue_warps(pair_tiles >= 4 * (num_sms() / 2)) == 4)
            gemm_step(Cfg<256, false, 4, true, 0, 2>{}, g);
        else if (pair && kb == 2)
            gemm_step(Cfg<256, false, 8, true, 0, 2>{}, g);
        else if (pair)
            gemm_step(Cfg<256, false, 8, true>{}, g);
        else if (L.bn == 256 && kb == 2)
            gemm_step(Cfg<256, false, 8, false, 0, 2>{}, g);
        else if (L.bn == 256)
            gemm_step(Cfg<256, false>{}, g);
        else if (kb == 2)
            gemm_step(Cfg<128, false, 8, false, 0, 2>{}, g);
        else
            gemm_step(Cfg<128, false>{}, g);
    }
    if (L.ksplit <= 1 || phase < 3) return set_last_error(PE_OK);
    const float* part = (const float*)((uint8_t*)ws + L.p_off);
    if (L.sk_q > 0) {
        GemmArgs gk = g;  // the reduction needs the k-iteration count of the GEMM
        gk.kiters = (int)((g.K + 128 / es - 1) / (128 / es));
        prog.push_back([part, out, L, plan, gk](cudaStream_t s) {
            return streamk_reduce_launch(part, out, L, &plan, gk, s);
        });
    } else {
        // launch_gemm rounds ksplit so that every unit gets >= 1 k-iteration
        const int kiters = (int)((g.K + 128 / es - 1) / (128 / es));
        int ks = g.ksplit;
        if (ks > 1 && kiters >= 2) {
            const int kper = (kiters + ks - 1) / ks;
            ks = (kiters + kper - 1) / kper;
        } else {
            ks = 1;
        }
        prog.push_back([part, out, L, plan, ks](cudaStream_t s) {
            return splitk_reduce_launch(part, out, L, &plan, ks, s);
        });
    }
    return set_last_error(PE_OK);
}

}  // namespace

#ifdef PE_STALL_STATS
// Diagnostic build only: copy (and clear) the per-CTA wait counters.
extern "C" int pe_stall_stats(unsigned long long* host, int n) {
    if (n > 1024 * 8) n = 1024 * 8;
    if (cudaMemcpyFromSymbol(host, pe_stall, n * sizeof(unsigned long long)) != cudaSuccess) return -1;
    static unsigned long long zero[1024 * 8];
    if (cudaMemcpyToSymbol(pe_stall, zero, sizeof(zero)) != cudaSuccess) return -1;
    return 0;
}
#endif

// Self-test of the bounded-wait path: one CTA waits on an mbarrier that nothing
// arrives on, through the same mbar_wait the GEMM pipeline uses, with a short
// limit. The wait gives up, records PE_ERR_TIMEOUT (site 15) in the device error
// word and the kernel returns normally, so the context stays usable.
__global__ void wait_timeout_probe(uint64_t timeout_ns, int* result) {
    __shared__ __align__(8) uint64_t bar;
    __shared__ int abort_sh;
    if (threadIdx.x == 0) {
        mbar_init(smem_u32(&bar), 1);
        abort_sh = 0;
        fence_barrier_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        const bool ok = mbar_wait(smem_u32(&bar), 0, &abort_sh, 15, timeout_ns);
        *result = ok ? 1 : 0;
    }
}

int wait_timeout_selftest(uint64_t timeout_ns, cudaStream_t s) {
    if (timeout_ns > 100000000ull) return set_last_error(PE_ERR_INVALID);  // at most 100 ms
    int* d = nullptr;
    int rc = check_cuda(cudaMallocAsync(&d, sizeof(int), s));
    if (rc) return rc;
    wait_timeout_probe<<<1, 32, 0, s>>>(timeout_ns, d);
    count_launch();
    int h = -1;
    rc = check_cuda(cudaGetLastError());
    if (!rc) rc = check_cuda(cudaMemcpyAsync(&h, d, sizeof(int), cudaMemcpyDeviceToHost, s));
    if (!rc) rc = check_cuda(cudaStreamSynchronize(s));
    cudaFreeAsync(d, s);
    if (rc) return rc;
    const int code = gemm_device_error(true);
    set_last_error(PE_OK);
    return h == 0 ? code : 0;  // the wait must not have succeeded
}

int gemm_device_error(bool clear) {
    int v = 0, zero = 0;
    if (cudaMemcpyFromSymbol(&v, g_device_error, sizeof(int)) != cudaSuccess) return -1;
    if (v && clear) cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int));
    return v;
}

}  // namespace pe
