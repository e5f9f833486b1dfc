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

// Tiled transpose: axis `ra` is unit-stride in the source, axis `wa` is
// unit-stride in the destination (ra != wa). Each block moves a 32x32 tile
// of the (wa, ra) plane for one combination of the remaining axes.
struct TileParams {
    int nd;
    int ra, wa;
    int64_t size[PE_MAX_RANK];
    int64_t sst[PE_MAX_RANK];
    int64_t dst[PE_MAX_RANK];
    int64_t tiles_r, tiles_w;      // tiles along ra / wa
    int64_t rest;                  // product of the other axes
};

template <typename T>
__global__ void __launch_bounds__(256) tiled_transpose(const T* __restrict__ src, T* __restrict__ dst,
                                                       TileParams p) {
    __shared__ T tile[32][33];
    const int64_t per_plane = p.tiles_r * p.tiles_w;
    const int64_t total = per_plane * p.rest;
    for (int64_t b = blockIdx.x; b < total; b += gridDim.x) {
        int64_t plane = b / per_plane;
        int64_t t = b - plane * per_plane;
        int64_t tw = t / p.tiles_r, tr = t - (t / p.tiles_r) * p.tiles_r;
        // decode the other axes
        int64_t so = 0, d = 0, rem = plane;
        for (int a = p.nd - 1; a >= 0; --a) {
            if (a == p.ra || a == p.wa) continue;
            int64_t q = rem / p.size[a];
            int64_t i = rem - q * p.size[a];
            rem = q;
            so += i * p.sst[a];
            d += i * p.dst[a];
        }
        const int64_t r0 = tr * 32, w0 = tw * 32;
        const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 8
        // read: consecutive threads walk the source-contiguous axis ra
        for (int k = ty; k < 32; k += 8) {
            int64_t r = r0 + tx, w = w0 + k;
            if (r < p.size[p.ra] && w < p.size[p.wa])
                tile[k][tx] = src[so + r * p.sst[p.ra] + w * p.sst[p.wa]];
        }
        __syncthreads();
        // write: consecutive threads walk the destination-contiguous axis wa
        for (int k = ty; k < 32; k += 8) {
            int64_t w = w0 + tx, r = r0 + k;
            if (r < p.size[p.ra] && w < p.size[p.wa])
                dst[d + r * p.dst[p.ra] + w * p.dst[p.wa]] = tile[tx][k];
        }
        __syncthreads();
    }
}

template <typename T>
int launch_copy(const void* src, void* dst, const CopyParams& cp, cudaStream_t s) {
    // find the unit-stride axes of source and destination
    int ra = -1, wa = -1;
    for (int a = 0; a < cp.nd; ++a) {
        if (cp.sst[a] == 1 && cp.size[a] > 1) ra = a;
        if (cp.dst[a] == 1 && cp.size[a] > 1) wa = a;
    }
    if (ra >= 0 && wa >= 0 && ra != wa && cp.size[ra] >= 8 && cp.size[wa] >= 8) {
        TileParams tp{};
        tp.nd = cp.nd;
        tp.ra = ra;
        tp.wa = wa;
        tp.rest = 1;
        for (int a = 0; a < cp.nd; ++a) {
            tp.size[a] = cp.size[a];
            tp.sst[a] = cp.sst[a];
            tp.dst[a] = cp.dst[a];
            if (a != ra && a != wa) tp.rest *= cp.size[a];
        }
        tp.tiles_r = (cp.size[ra] + 31) / 32;
        tp.tiles_w = (cp.size[wa] + 31) / 32;
        int64_t blocks = tp.tiles_r * tp.tiles_w * tp.rest;
        int64_t cap = (int64_t)num_sms() * 16;
        tiled_transpose<T><<<(int)(blocks < cap ? blocks : cap), 256, 0, s>>>((const T*)src, (T*)dst,
                                                                            tp);
    } else {
        int64_t blocks = (cp.n + 255) / 256;
        int64_t cap = (int64_t)num_sms() * 8;
        strided_copy<T><<<(int)(blocks < cap ? blocks : cap), 256, 0, s>>>((const T*)src, (T*)dst,
                                                                          cp);
    }
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
