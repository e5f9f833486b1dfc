// pe_stream.cu - Hadamard and broadcast multiplies as 128-bit streaming kernels.
//
// Replaces the Ascend Vector kernels of include/pto_einsum_elementwise.h
// (elementwise_mul:27-127, broadcast_mul:129-370). Each thread moves 16 bytes
// of every input per step (float4, or 8 x half) with streaming cache hints and
// writes fp32 results with 16-byte stores; a scalar tail loop covers the
// ragged end and unaligned buffers. Products are formed as
// float(a) * float(b), the same single rounding as cpu_einsum.h:87-92, so the
// results are bit-identical to the CPU reference.
#include <cuda_fp16.h>

#include "pe_common.cuh"

namespace pe {

namespace {

__device__ __forceinline__ float4 ld_stream(const float4* p) { return __ldcs(p); }
__device__ __forceinline__ uint4 ld_stream(const uint4* p) { return __ldcs(p); }
__device__ __forceinline__ void st_stream(float4* p, float4 v) { __stcs(p, v); }

__device__ __forceinline__ void unpack8(const uint4& v, float (&f)[8]) {
    const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        float2 t = __half22float2(h[i]);
        f[2 * i] = t.x;
        f[2 * i + 1] = t.y;
    }
}

__device__ __forceinline__ float to_f(float x) { return x; }

// Lane l holds the 8 fp32 results of elements [8l, 8l+8) of a warp's
// 256-element block starting at `base`. Storing them directly would make each
// 16-byte store instruction cover only half of every 32-byte sector it
// touches; instead lanes exchange values so that each of the two store
// instructions writes 512 contiguous bytes (lane l writes elements 4l..4l+3,
// then 128+4l..).
__device__ __forceinline__ void store8_coalesced(float* __restrict__ base, const float (&p)[8], int lane) {
#pragma unroll
    for (int half = 0; half < 2; ++half) {
        const int src = half * 16 + (lane >> 1);
        const bool hi = lane & 1;
        float q[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const float lo_v = __shfl_sync(0xffffffffu, p[k], src);
            const float hi_v = __shfl_sync(0xffffffffu, p[4 + k], src);
            q[k] = hi ? hi_v : lo_v;
        }
        st_stream(reinterpret_cast<float4*>(base) + half * 32 + lane, make_float4(q[0], q[1], q[2], q[3]));
    }
}
__device__ __forceinline__ float to_f(__half x) { return __half2float(x); }

// ---- Hadamard -----------------------------------------------------------------
__global__ void __launch_bounds__(256) ew_mul_f32_vec(const float4* __restrict__ a,
                                                      const float4* __restrict__ b,
                                                      float4* __restrict__ out, int64_t nvec) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t step = (int64_t)gridDim.x * blockDim.x;
    for (; i + step < nvec; i += 2 * step) {
        float4 x0 = ld_stream(a + i), y0 = ld_stream(b + i);
        float4 x1 = ld_stream(a + i + step), y1 = ld_stream(b + i + step);
        st_stream(out + i, make_float4(x0.x * y0.x, x0.y * y0.y, x0.z * y0.z, x0.w * y0.w));
        st_stream(out + i + step, make_float4(x1.x * y1.x, x1.y * y1.y, x1.z * y1.z, x1.w * y1.w));
    }
    if (i < nvec) {
        float4 x0 = ld_stream(a + i), y0 = ld_stream(b + i);
        st_stream(out + i, make_float4(x0.x * y0.x, x0.y * y0.y, x0.z * y0.z, x0.w * y0.w));
    }
}

__device__ __forceinline__ void mul8(const uint4& a, const uint4& b, float (&p)[8]) {
    float x[8], y[8];
    unpack8(a, x);
    unpack8(b, y);
#pragma unroll
    for (int k = 0; k < 8; ++k) p[k] = x[k] * y[k];
}

// Stores the 8 products of vector i: warp-cooperatively when the warp's 32
// consecutive vectors are all in range, else one thread at a time.
__device__ __forceinline__ void store8(float* __restrict__ out, int64_t i, int lane, bool full_warp,
                                       const float (&p)[8]) {
    if (full_warp) {
        store8_coalesced(out + (i - lane) * 8, p, lane);
    } else {
        float4* o = reinterpret_cast<float4*>(out) + 2 * i;
        st_stream(o, make_float4(p[0], p[1], p[2], p[3]));
        st_stream(o + 1, make_float4(p[4], p[5], p[6], p[7]));
    }
}

__global__ void __launch_bounds__(256) ew_mul_f16_vec(const uint4* __restrict__ a,
                                                      const uint4* __restrict__ b,
                                                      float* __restrict__ out, int64_t nvec) {
    const int lane = threadIdx.x & 31;
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t step = (int64_t)gridDim.x * blockDim.x;
    // four vectors of each operand in flight per thread
    for (; i < nvec; i += 4 * step) {
        uint4 x[4], y[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const int64_t iq = i + q * step;
            x[q] = iq < nvec ? ld_stream(a + iq) : make_uint4(0, 0, 0, 0);
            y[q] = iq < nvec ? ld_stream(b + iq) : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const int64_t iq = i + q * step;
            if (iq < nvec) {
                float p[8];
                mul8(x[q], y[q], p);
                store8(out, iq, lane, iq - lane + 32 <= nvec, p);
            }
        }
    }
}

template <typename T>
__global__ void ew_mul_scalar(const T* __restrict__ a, const T* __restrict__ b,
                              float* __restrict__ out, int64_t begin, int64_t n) {
    int64_t i = begin + (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t step = (int64_t)gridDim.x * blockDim.x;
    for (; i < n; i += step) out[i] = to_f(a[i]) * to_f(b[i]);
}

// ---- broadcast ----------------------------------------------------------------
struct BcastParams {
    int64_t n;         // elements of the output / full operand
    int mode;          // 0 column-expand, 1 scalar per group
    int outer_rank;
    FastDiv inner_v;   // Inner / VEC  (vector path) or Inner (scalar path)
    FastDiv cc_v;      // Cc / VEC or Cc
    FastDiv odiv[PE_MAX_RANK];    // product of outer dims inside axis q
    FastDiv odim[PE_MAX_RANK];    // outer dim q
    int64_t obstride[PE_MAX_RANK];
};

__device__ __forceinline__ int64_t outer_base(const BcastParams& p, uint32_t o) {
    int64_t base = 0;
    for (int q = 0; q < p.outer_rank; ++q) {
        uint32_t t = fdiv(o, p.odiv[q]);
        uint32_t idx = t - fdiv(t, p.odim[q]) * p.odim[q].div;
        base += (int64_t)idx * p.obstride[q];
    }
    return base;
}

template <typename T>
__device__ __forceinline__ void bcast_apply(const T* __restrict__ bc, float* __restrict__ out,
                                            const BcastParams& p, uint32_t v, const uint4& raw, int lane,
                                            bool full_warp) {
    constexpr int VEC = 16 / sizeof(T);
    uint32_t o = fdiv(v, p.inner_v);
    uint32_t w = v - o * p.inner_v.div;  // vector index inside the group
    int64_t boff = outer_base(p, o);
    float x[VEC], y[VEC];
    if constexpr (sizeof(T) == 4) {
        x[0] = __uint_as_float(raw.x); x[1] = __uint_as_float(raw.y);
        x[2] = __uint_as_float(raw.z); x[3] = __uint_as_float(raw.w);
    } else {
        unpack8(raw, x);
    }
    if (p.mode == 0) {
        uint32_t c = w - fdiv(w, p.cc_v) * p.cc_v.div;
        const uint4 b4 = __ldg(reinterpret_cast<const uint4*>(bc + boff + (int64_t)c * VEC));
        if constexpr (sizeof(T) == 4) {
            y[0] = __uint_as_float(b4.x); y[1] = __uint_as_float(b4.y);
            y[2] = __uint_as_float(b4.z); y[3] = __uint_as_float(b4.w);
        } else {
            unpack8(b4, y);
        }
    } else {
        float sc = to_f(bc[boff]);
#pragma unroll
        for (int j = 0; j < VEC; ++j) y[j] = sc;
    }
    float r[VEC];
#pragma unroll
    for (int j = 0; j < VEC; ++j) r[j] = x[j] * y[j];
    if constexpr (VEC == 8) {
        store8(out, v, lane, full_warp, r);
    } else {
        st_stream(reinterpret_cast<float4*>(out) + v, make_float4(r[0], r[1], r[2], r[3]));
    }
}

// Vector path: Inner and Cc are multiples of VEC, so a vector never crosses a
// group and (mode 0) the matching broadcast run is VEC contiguous elements.
// Each iteration issues four independent 16-byte loads of the full operand
// before using any, to keep more bytes in flight per thread.
template <typename T>
__global__ void __launch_bounds__(256) bcast_mul_vec(const T* __restrict__ full,
                                                     const T* __restrict__ bc,
                                                     float* __restrict__ out, BcastParams p) {
    constexpr int VEC = 16 / sizeof(T);
    const int lane = threadIdx.x & 31;
    const uint32_t nvec = (uint32_t)(p.n / VEC);
    const uint32_t step = gridDim.x * blockDim.x;
    const uint4* src = reinterpret_cast<const uint4*>(full);
    for (uint32_t v = blockIdx.x * blockDim.x + threadIdx.x; v < nvec; v += 4 * step) {
        uint4 a[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const uint32_t vq = v + q * step;
            a[q] = vq < nvec ? ld_stream(src + vq) : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const uint32_t vq = v + q * step;
            if (vq < nvec) bcast_apply<T>(bc, out, p, vq, a[q], lane, (int64_t)vq - lane + 32 <= (int64_t)nvec);
        }
    }
}

// Generic path: one element per thread step, any alignment. Offsets use 64-bit
// division, so it is only taken for shapes the vector path cannot cover.
struct BcastGeneric {
    int64_t n, inner, cc;
    int mode, outer_rank;
    int64_t odiv[PE_MAX_RANK], odim[PE_MAX_RANK], obstride[PE_MAX_RANK];
};

template <typename T>
__global__ void bcast_mul_scalar(const T* __restrict__ full, const T* __restrict__ bc,
                                 float* __restrict__ out, BcastGeneric p) {
    int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t step = (int64_t)gridDim.x * blockDim.x;
    for (; e < p.n; e += step) {
        int64_t o = e / p.inner;
        int64_t boff = 0;
        for (int q = 0; q < p.outer_rank; ++q) boff += ((o / p.odiv[q]) % p.odim[q]) * p.obstride[q];
        if (p.mode == 0) boff += (e % p.inner) % p.cc;
        out[e] = to_f(full[e]) * to_f(bc[boff]);
    }
}

int grid_for(int64_t work, int threads) {
    int64_t blocks = (work + threads - 1) / threads;
    int64_t cap = (int64_t)num_sms() * 8;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    return (int)blocks;
}

inline bool aligned16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

}  // namespace

int elementwise_mul(int32_t dtype, const void* a, const void* b, float* out, int64_t n,
                    cudaStream_t s) {
    if (n < 0 || (n > 0 && (!a || !b || !out))) return set_last_error(PE_ERR_INVALID);
    if (dtype != PE_F32 && dtype != PE_F16) return set_last_error(PE_ERR_INVALID);
    if (n == 0) return set_last_error(PE_OK);
    const int es = dtype == PE_F32 ? 4 : 2;
    const int vec = 16 / es;
    int64_t nvec = (aligned16(a) && aligned16(b) && aligned16(out)) ? n / vec : 0;
    if (nvec > 0) {
        if (dtype == PE_F32)
            ew_mul_f32_vec<<<grid_for((nvec + 1) / 2, 256), 256, 0, s>>>(
                (const float4*)a, (const float4*)b, (float4*)out, nvec);
        else
            ew_mul_f16_vec<<<grid_for((nvec + 3) / 4, 256), 256, 0, s>>>((const uint4*)a, (const uint4*)b,
                                                                         out, nvec);
        count_launch();
    }
    int64_t done = nvec * vec;
    if (done < n) {
        if (dtype == PE_F32)
            ew_mul_scalar<float><<<grid_for(n - done, 256), 256, 0, s>>>(
                (const float*)a, (const float*)b, out, done, n);
        else
            ew_mul_scalar<__half><<<grid_for(n - done, 256), 256, 0, s>>>(
                (const __half*)a, (const __half*)b, out, done, n);
        count_launch();
    }
    return check_cuda(cudaGetLastError());
}

int broadcast_mul(const pe_broadcast_plan* pl, const void* full, const void* bc, float* out,
                  cudaStream_t s) {
    if (!pl || (pl->dtype != PE_F32 && pl->dtype != PE_F16) || pl->outer_rank < 0 ||
        pl->outer_rank > PE_MAX_RANK || pl->n < 0)
        return set_last_error(PE_ERR_INVALID);
    if (pl->n == 0) return set_last_error(PE_OK);
    if (!full || !bc || !out) return set_last_error(PE_ERR_INVALID);
    const int es = pl->dtype == PE_F32 ? 4 : 2;
    const int vec = 16 / es;
    const int64_t inner = pl->Inner > 0 ? pl->Inner : 1;
    const int64_t cc = pl->Cc > 0 ? pl->Cc : 1;
    bool vec_ok = aligned16(full) && aligned16(out) && pl->n % vec == 0 && inner % vec == 0 &&
                  pl->n / vec < (1ll << 32) && pl->n / inner < (1ll << 32);
    if (pl->mode == 0) vec_ok = vec_ok && cc % vec == 0 && aligned16(bc);
    for (int q = 0; q < pl->outer_rank && vec_ok; ++q)
        if (pl->mode == 0 && pl->outer_bstride[q] % vec) vec_ok = false;
    if (vec_ok) {
        BcastParams p{};
        p.n = pl->n;
        p.mode = pl->mode;
        p.outer_rank = pl->outer_rank;
        p.inner_v = make_fastdiv((uint32_t)(inner / vec));
        p.cc_v = make_fastdiv((uint32_t)(cc / vec));
        int64_t run = 1;
        for (int q = pl->outer_rank - 1; q >= 0; --q) {
            p.odiv[q] = make_fastdiv((uint32_t)run);
            p.odim[q] = make_fastdiv((uint32_t)pl->outer_dims[q]);
            p.obstride[q] = pl->outer_bstride[q];
            run *= pl->outer_dims[q];
        }
        int64_t nvec = pl->n / vec;
        if (pl->dtype == PE_F32)
            bcast_mul_vec<float><<<grid_for((nvec + 3) / 4, 256), 256, 0, s>>>((const float*)full,
                                                                    (const float*)bc, out, p);
        else
            bcast_mul_vec<__half><<<grid_for((nvec + 3) / 4, 256), 256, 0, s>>>((const __half*)full,
                                                                     (const __half*)bc, out, p);
    } else {
        BcastGeneric p{};
        p.n = pl->n;
        p.inner = inner;
        p.cc = cc;
        p.mode = pl->mode;
        p.outer_rank = pl->outer_rank;
        int64_t run = 1;
        for (int q = pl->outer_rank - 1; q >= 0; --q) {
            p.odiv[q] = run;
            p.odim[q] = pl->outer_dims[q] > 0 ? pl->outer_dims[q] : 1;
            p.obstride[q] = pl->outer_bstride[q];
            run *= p.odim[q];
        }
        if (pl->dtype == PE_F32)
            bcast_mul_scalar<float><<<grid_for(pl->n, 256), 256, 0, s>>>((const float*)full,
                                                                        (const float*)bc, out, p);
        else
            bcast_mul_scalar<__half><<<grid_for(pl->n, 256), 256, 0, s>>>(
                (const __half*)full, (const __half*)bc, out, p);
    }
    count_launch();
    return check_cuda(cudaGetLastError());
}

}  // namespace pe
