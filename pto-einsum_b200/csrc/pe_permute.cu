// pe_permute.cu - N-D permute / strided gather.
//
// Replaces the Ascend transpose family (include/pto_einsum_transpose.h:19-678)
// for the plans TMA tensor maps cannot read directly, and backs the standalone
// run_transpose_* entry points. A logical index space of up to PE_MAX_RANK
// axes is walked in destination order; each axis has a source and destination
// stride, so one kernel covers plain permutes (transpose.h T4-T7), K-padded
// destinations (T2/T3) and gathers into the canonical [batch, free, contract]
// layout. When the source's innermost axis is not the destination's innermost
// axis the kernel stages 32x32 tiles through shared memory so both the global
// reads and the global writes are coalesced.
#include <cuda_fp16.h>

#include "pe_common.cuh"
#include "pe_internal.h"

namespace pe {

namespace {

struct CopyParams {
    int nd;                        // logical axes (outermost first)
    int64_t size[PE_MAX_RANK];
    int64_t sst[PE_MAX_RANK];      // source element strides
    int64_t dst[PE_MAX_RANK];      // destination element strides
    int64_t n;                     // product of sizes
};

template <typename T>
__global__ void __launch_bounds__(256) strided_copy(const T* __restrict__ src, T* __restrict__ dst,
                                                    CopyParams p) {
    int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t step = (int64_t)gridDim.x * blockDim.x;
    for (; e < p.n; e += step) {
        int64_t rem = e, so = 0, d = 0;
        for (int a = p.nd - 1; a >= 0; --a) {
            int64_t q = rem / p.size[a];
            int64_t i = rem - q * p.size[a];
            rem = q;
            so += i * p.sst[a];
            d += i * p.dst[a];
        }
        dst[d] = src[so];
    }
}

// Run copy: the innermost logical axis is unit-stride in both source and
// destination, so whole runs of it are copied with 16-byte vectors; the outer
// axes are decoded once per vector with multiply-high division.
struct RunParams {
    int nd;                          // outer axes (outermost first)
    FastDiv div[PE_MAX_RANK];
    int64_t sst[PE_MAX_RANK], dst[PE_MAX_RANK];
    FastDiv rv;                      // vectors per run
    uint32_t nvec;
};

template <typename T>
__global__ void __launch_bounds__(256) run_copy(const T* __restrict__ src, T* __restrict__ dst, RunParams p) {
    constexpr int VEC = 16 / sizeof(T);
    const uint32_t step = gridDim.x * blockDim.x;
    for (uint32_t v = blockIdx.x * blockDim.x + threadIdx.x; v < p.nvec; v += step) {
        uint32_t row = fdiv(v, p.rv);
        const uint32_t c = v - row * p.rv.div;
        int64_t so = (int64_t)c * VEC, d = (int64_t)c * VEC;
        for (int a = p.nd - 1; a >= 0; --a) {
            const uint32_t q = fdiv(row, p.div[a]);
            const uint32_t idx = row - q * p.div[a].div;
            row = q;
            so += (int64_t)idx * p.sst[a];
            d += (int64_t)idx * p.dst[a];
        }
        *reinterpret_cast<uint4*>(dst + d) = __ldcs(reinterpret_cast<const uint4*>(src + so));
    }
}

// TDxTD tiled transpose with 16-byte global accesses on both sides: axis ra
// is unit-stride in the source, wa in the destination. When sizes, strides and
// bases allow 16-byte vectors every tile (edge tiles included, bounds checked
// per vector) takes the vector path; otherwise element copies.
struct TileTParams {
    int nd, ra, wa;
    uint32_t skip;                   // axes not decoded per tile (ra, wa and their partners)
    int64_t size[PE_MAX_RANK], sst[PE_MAX_RANK], dst[PE_MAX_RANK];
    int64_t nr, nw;                  // tile-space extents (ra or wa times its partner)
    FastDiv rlo, wlo;                // extent of ra / wa inside the combined index
    int64_t sw, sw_hi;               // source strides of wa and of its partner
    int64_t dr, dr_hi;               // destination strides of ra and of its partner
    int64_t tiles_r, tiles_w, rest;
    int vec_ok;
};

// Source offset of tile-space row w, destination offset of tile-space row r.
template <bool G>
__device__ __forceinline__ int64_t src_row(const TileTParams& p, int64_t w) {
    if (!G) return w * p.sw;
    const uint32_t hi = fdiv((uint32_t)w, p.wlo);
    return (int64_t)hi * p.sw_hi + (w - (int64_t)hi * p.wlo.div) * p.sw;
}
template <bool G>
__device__ __forceinline__ int64_t dst_row(const TileTParams& p, int64_t r) {
    if (!G) return r * p.dr;
    const uint32_t hi = fdiv((uint32_t)r, p.rlo);
    return (int64_t)hi * p.dr_hi + (r - (int64_t)hi * p.rlo.div) * p.dr;
}

template <typename T, int TD, bool G>
__global__ void __launch_bounds__(256, 8) tile_transpose(const T* __restrict__ src, T* __restrict__ dst,
                                                      TileTParams p) {
    constexpr int VEC = 16 / sizeof(T);
    constexpr int PAD = 4 / sizeof(T);           // one 32-bit word of padding per row
    constexpr int VPR = TD / VEC;                // vectors per tile row
    __shared__ T tile[TD][TD + PAD];             // tile[w][r]
    const int64_t per_plane = p.tiles_r * p.tiles_w;
    const int64_t total = per_plane * p.rest;
    const int64_t nr = p.nr, nw = p.nw;
    for (int64_t b = blockIdx.x; b < total; b += gridDim.x) {
        const int64_t plane = b / per_plane, t = b - plane * per_plane;
        const int64_t tw = t / p.tiles_r, tr = t - tw * p.tiles_r;
        int64_t so = 0, d = 0, rem = plane;
        for (int a = p.nd - 1; a >= 0; --a) {
            if ((p.skip >> a) & 1) continue;
            const int64_t q = rem / p.size[a];
            const int64_t idx = rem - q * p.size[a];
            rem = q;
            so += idx * p.sst[a];
            d += idx * p.dst[a];
        }
        const int64_t r0 = (int64_t)tr * TD, w0 = (int64_t)tw * TD;
        if (p.vec_ok) {
            // read: rows w, TD consecutive r as 16-byte vectors
#pragma unroll 4
            for (int k = threadIdx.x; k < TD * VPR; k += 256) {
                const int w = k / VPR, rv = k % VPR;
                if (w0 + w < nw && r0 + rv * VEC < nr) {
                    const uint4 x = __ldcs(reinterpret_cast<const uint4*>(src + so + src_row<G>(p, w0 + w) + r0 + rv * VEC));
                    const T* e = reinterpret_cast<const T*>(&x);
#pragma unroll
                    for (int q = 0; q < VEC; ++q) tile[w][rv * VEC + q] = e[q];
                }
            }
            __syncthreads();
            // write: rows r, TD consecutive w as 16-byte vectors
#pragma unroll 4
            for (int k = threadIdx.x; k < TD * VPR; k += 256) {
                const int r = k / VPR, wv = k % VPR;
                if (r0 + r < nr && w0 + wv * VEC < nw) {
                    uint4 y;
                    T* e = reinterpret_cast<T*>(&y);
#pragma unroll
                    for (int q = 0; q < VEC; ++q) e[q] = tile[wv * VEC + q][r];
                    *reinterpret_cast<uint4*>(dst + d + dst_row<G>(p, r0 + r) + w0 + wv * VEC) = y;
                }
            }
        } else {
            for (int k = threadIdx.x; k < TD * TD; k += 256) {
                const int w = k / TD, r = k % TD;
                if (r0 + r < nr && w0 + w < nw) tile[w][r] = src[so + src_row<G>(p, w0 + w) + r0 + r];
            }
            __syncthreads();
            for (int k = threadIdx.x; k < TD * TD; k += 256) {
                const int r = k / TD, w = k % TD;
                if (r0 + r < nr && w0 + w < nw) dst[d + dst_row<G>(p, r0 + r) + w0 + w] = tile[w][r];
            }
        }
        __syncthreads();
    }
}

// 2-byte transpose, 128x128 tiles: each thread loads the same 16-byte column
// slice of two neighbouring source rows (w, w+1) and packs element pairs into
// 32-bit words, so shared memory holds tile[r][w/2] as words. The 16-byte
// chunks of each shared row are XOR-swizzled by r/8, which keeps both the
// packed word stores and the 16-byte chunk loads of the write side free of
// bank conflicts. Requires the TileTParams vector conditions (vec_ok).
template <bool G>
__global__ void __launch_bounds__(256) tile_transpose_h128(const uint16_t* __restrict__ src,
                                                           uint16_t* __restrict__ dst, TileTParams p) {
    __shared__ __align__(16) uint32_t tile[128][64];
    const int64_t per_plane = p.tiles_r * p.tiles_w;
    const int64_t total = per_plane * p.rest;
    const int64_t nr = p.nr, nw = p.nw;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int64_t b = blockIdx.x; b < total; b += gridDim.x) {
        const int64_t plane = b / per_plane, t = b - plane * per_plane;
        const int64_t tw = t / p.tiles_r, tr = t - tw * p.tiles_r;
        int64_t so = 0, d = 0, rem = plane;
        for (int a = p.nd - 1; a >= 0; --a) {
            if ((p.skip >> a) & 1) continue;
            const int64_t q = rem / p.size[a];
            const int64_t idx = rem - q * p.size[a];
            rem = q;
            so += idx * p.sst[a];
            d += idx * p.dst[a];
        }
        const int64_t r0 = tr * 128, w0 = tw * 128;
        // read side: 64 row pairs x 16 column vectors = 1024 items, 4 per thread;
        // a warp covers 8 column vectors (128 B) of 4 row pairs
#pragma unroll
        for (int it = 0; it < 4; ++it) {
            const int idx = it * 8 + warp;                    // 0..31
            const int rv = (idx & 1) * 8 + (lane & 7);        // column vector 0..15
            const int wp = (idx >> 1) * 4 + (lane >> 3);      // row pair 0..63
            const int64_t w = w0 + 2 * wp;
            if (w < nw && r0 + rv * 8 < nr) {
                const uint16_t* sp = src + so + src_row<G>(p, w) + r0 + rv * 8;
                const uint4 x0 = __ldcs(reinterpret_cast<const uint4*>(sp));
                const uint4 x1 = __ldcs(reinterpret_cast<const uint4*>(sp + p.sw));
                const uint32_t a[4] = {x0.x, x0.y, x0.z, x0.w}, c[4] = {x1.x, x1.y, x1.z, x1.w};
                const int chunk = ((wp >> 2) ^ rv) * 4 + (wp & 3);
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    tile[rv * 8 + 2 * q][chunk] = __byte_perm(a[q], c[q], 0x5410);
                    tile[rv * 8 + 2 * q + 1][chunk] = __byte_perm(a[q], c[q], 0x7632);
                }
            }
        }
        __syncthreads();
        // write side: 128 rows x 16 chunks of 8 elements, 8 per thread
#pragma unroll
        for (int it = 0; it < 8; ++it) {
            const int k = it * 256 + threadIdx.x;
            const int r = k >> 4, cw = k & 15;
            if (r0 + r < nr && w0 + cw * 8 < nw) {
                const uint4 y = *reinterpret_cast<const uint4*>(&tile[r][(cw ^ (r >> 3)) * 4]);
                *reinterpret_cast<uint4*>(dst + d + dst_row<G>(p, r0 + r) + w0 + cw * 8) = y;
            }
        }
        __syncthreads();
    }
}

template <typename T>
int launch_copy(const void* src, void* dst, const CopyParams& cp, cudaStream_t s) {
    constexpr int VEC = 16 / sizeof(T);
    const bool al = ((uintptr_t)src % 16 == 0) && ((uintptr_t)dst % 16 == 0);
    const int last = cp.nd - 1;
    // (1) innermost axis unit-stride on both sides: vectorised run copy
    if (al && cp.nd >= 1 && cp.sst[last] == 1 && cp.dst[last] == 1 && cp.size[last] % VEC == 0 &&
        cp.n / VEC < (1ll << 31)) {
        bool ok = true;
        RunParams rp{};
        rp.nd = cp.nd - 1;
        for (int a = 0; a < rp.nd; ++a) {
            if (cp.sst[a] % VEC || cp.dst[a] % VEC || cp.size[a] >= (1ll << 32)) ok = false;
            rp.div[a] = make_fastdiv((uint32_t)cp.size[a]);
            rp.sst[a] = cp.sst[a];
            rp.dst[a] = cp.dst[a];
        }
        if (ok) {
            rp.rv = make_fastdiv((uint32_t)(cp.size[last] / VEC));
            rp.nvec = (uint32_t)(cp.n / VEC);
            int64_t blocks = ((int64_t)rp.nvec + 255) / 256, cap = (int64_t)num_sms() * 8;
            run_copy<T><<<(int)(blocks < cap ? blocks : cap), 256, 0, s>>>((const T*)src, (T*)dst, rp);
            count_launch();
            return check_cuda(cudaGetLastError());
        }
    }
    // find the unit-stride axes of source and destination
    int ra = -1, wa = -1;
    for (int a = 0; a < cp.nd; ++a) {
        if (cp.sst[a] == 1 && cp.size[a] > 1) ra = a;
        if (cp.dst[a] == 1 && cp.size[a] > 1) wa = a;
    }
    // (2) transpose of the unit-stride axis: square tiles through shared memory
    if (ra >= 0 && wa >= 0 && ra != wa && cp.size[ra] >= 8 && cp.size[wa] >= 8) {
        TileTParams tp{};
        tp.nd = cp.nd;
        tp.ra = ra;
        tp.wa = wa;
        // A narrow unit-stride axis is widened by the axis that continues it
        // contiguously on the same side (destination for wa, source for ra),
        // so tiles stay full.
        int wp = -1, rp = -1;
        for (int a = 0; a < cp.nd; ++a) {
            if (a == ra || a == wa) continue;
            if (cp.size[wa] < 128 && wp < 0 && cp.dst[a] == cp.size[wa]) wp = a;
        }
        for (int a = 0; a < cp.nd; ++a) {
            if (a == ra || a == wa || a == wp) continue;
            if (cp.size[ra] < 128 && rp < 0 && cp.sst[a] == cp.size[ra]) rp = a;
        }
        tp.nw = cp.size[wa] * (wp >= 0 ? cp.size[wp] : 1);
        tp.nr = cp.size[ra] * (rp >= 0 ? cp.size[rp] : 1);
        if (tp.nw < (1ll << 31) && tp.nr < (1ll << 31)) {
            tp.wlo = make_fastdiv((uint32_t)cp.size[wa]);
            tp.rlo = make_fastdiv((uint32_t)cp.size[ra]);
            tp.sw = cp.sst[wa];
            tp.sw_hi = wp >= 0 ? cp.sst[wp] : 0;
            tp.dr = cp.dst[ra];
            tp.dr_hi = rp >= 0 ? cp.dst[rp] : 0;
            tp.skip = (1u << ra) | (1u << wa) | (wp >= 0 ? 1u << wp : 0u) | (rp >= 0 ? 1u << rp : 0u);
            tp.rest = 1;
            bool vec = al && cp.size[ra] % VEC == 0 && cp.size[wa] % VEC == 0;
            for (int a = 0; a < cp.nd; ++a) {
                tp.size[a] = cp.size[a];
                tp.sst[a] = cp.sst[a];
                tp.dst[a] = cp.dst[a];
                if (!((tp.skip >> a) & 1)) tp.rest *= cp.size[a];
                if (a != ra && cp.sst[a] % VEC) vec = false;
                if (a != wa && cp.dst[a] % VEC) vec = false;
            }
            tp.vec_ok = vec ? 1 : 0;
            const bool big = sizeof(T) == 2 && vec && tp.nr >= 128 && tp.nw >= 128;
            const int td = big ? 128 : 64;
            tp.tiles_r = (tp.nr + td - 1) / td;
            tp.tiles_w = (tp.nw + td - 1) / td;
            int64_t blocks = tp.tiles_r * tp.tiles_w * tp.rest;
            int64_t cap = (int64_t)num_sms() * 16;
            const int g = (int)(blocks < cap ? blocks : cap);
            const bool grouped = wp >= 0 || rp >= 0;
            if constexpr (sizeof(T) == 2) {
                // 2-byte elements use packed 128x128 tiles when both extents fill them
                if (big) {
                    if (grouped)
                        tile_transpose_h128<true><<<g, 256, 0, s>>>((const uint16_t*)src, (uint16_t*)dst, tp);
                    else
                        tile_transpose_h128<false><<<g, 256, 0, s>>>((const uint16_t*)src, (uint16_t*)dst, tp);
                } else if (grouped) {
                    tile_transpose<T, 64, true><<<g, 256, 0, s>>>((const T*)src, (T*)dst, tp);
                } else {
                    tile_transpose<T, 64, false><<<g, 256, 0, s>>>((const T*)src, (T*)dst, tp);
                }
            } else if (grouped) {
                tile_transpose<T, 64, true><<<g, 256, 0, s>>>((const T*)src, (T*)dst, tp);
            } else {
                tile_transpose<T, 64, false><<<g, 256, 0, s>>>((const T*)src, (T*)dst, tp);
            }
            count_launch();
            return check_cuda(cudaGetLastError());
        }
    }
    // (3) anything else: one element per thread step
    int64_t blocks = (cp.n + 255) / 256;
    int64_t cap = (int64_t)num_sms() * 8;
    strided_copy<T><<<(int)(blocks < cap ? blocks : cap), 256, 0, s>>>((const T*)src, (T*)dst, cp);
    count_launch();
    return check_cuda(cudaGetLastError());
}

}  // namespace

int strided_copy_launch(int es, int nd, const int64_t* size, const int64_t* sst, const int64_t* dst_st,
                        const void* src, void* dst, cudaStream_t s) {
    CopyParams cp{};
    cp.n = 1;
    // drop size-1 axes (their index is always 0)
    for (int a = 0; a < nd; ++a) {
        if (size[a] == 0) return set_last_error(PE_OK);
        if (size[a] == 1) continue;
        cp.size[cp.nd] = size[a];
        cp.sst[cp.nd] = sst[a];
        cp.dst[cp.nd] = dst_st[a];
        cp.nd++;
        cp.n *= size[a];
    }
    // merge neighbours that are contiguous in both source and destination
    {
        int k = 0;
        for (int a = 0; a < cp.nd; ++a) {
            if (k > 0 && cp.sst[k - 1] == cp.sst[a] * cp.size[a] && cp.dst[k - 1] == cp.dst[a] * cp.size[a]) {
                cp.size[k - 1] *= cp.size[a];
                cp.sst[k - 1] = cp.sst[a];
                cp.dst[k - 1] = cp.dst[a];
            } else {
                cp.size[k] = cp.size[a];
                cp.sst[k] = cp.sst[a];
                cp.dst[k] = cp.dst[a];
                ++k;
            }
        }
        cp.nd = k;
    }
    if (cp.nd == 0) {
        cp.nd = 1;
        cp.size[0] = 1;
        cp.sst[0] = cp.dst[0] = 0;
    }
    if (es == 4) return launch_copy<float>(src, dst, cp, s);
    if (es == 2) return launch_copy<uint16_t>(src, dst, cp, s);
    return set_last_error(PE_ERR_INVALID);
}

int permute(const pe_permute_plan* pl, const void* in, void* out, cudaStream_t s) {
    if (!pl || pl->dims < 0 || pl->dims > PE_MAX_RANK || (pl->dtype != PE_F32 && pl->dtype != PE_F16))
        return set_last_error(PE_ERR_INVALID);
    int64_t st[PE_MAX_RANK], size[PE_MAX_RANK], sst[PE_MAX_RANK], dst[PE_MAX_RANK];
    int64_t run = 1, n = 1;
    for (int a = pl->dims - 1; a >= 0; --a) {
        st[a] = run;
        run *= pl->from_shape[a];
    }
    bool seen[PE_MAX_RANK] = {false};
    for (int a = 0; a < pl->dims; ++a) {
        int p = pl->perm[a];
        if (p < 0 || p >= pl->dims || seen[p]) return set_last_error(PE_ERR_INVALID);
        seen[p] = true;
        size[a] = pl->from_shape[p];
        sst[a] = st[p];
        n *= size[a];
    }
    run = 1;
    for (int a = pl->dims - 1; a >= 0; --a) {
        dst[a] = run;
        run *= size[a];
    }
    if (n == 0) return set_last_error(PE_OK);
    if (!in || !out) return set_last_error(PE_ERR_INVALID);
    return strided_copy_launch(pl->dtype == PE_F32 ? 4 : 2, pl->dims, size, sst, dst, in, out, s);
}

}  // namespace pe
