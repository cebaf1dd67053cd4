// Fused elementwise ops of a decoder layer (engine/model.py:41-72,
// engine/qwen.py:43-75) for 16-bit models: RMSNorm (optionally after the
// residual add), rotate-half RoPE of q and k in place, and the SwiGLU gate.
// Each replaces a chain of small framework kernels with one launch and
// reproduces the chain's rounding: every elementwise step of the chain rounds
// to the model dtype exactly where the chain does.
//
//   rmsnorm:  xf = float(x); r = sqrt(mean(xf^2) + eps); out = T((xf / r) * float(w))
//             (engine/model.py RMSNorm.forward).  The mean is a fixed-order
//             block sum times fl(1/dim), so it may differ from another sum
//             order in the last fp32 bit.
//   add_rmsnorm: h' = T(float(h) + float(d)) (the residual add), then rmsnorm(h').
//   rope:     x' = T(T(x * c) + T(rh(x) * s)), rh(x) = (-x[d/2:], x[:d/2])
//             (engine/model.py:50-56: apply_rotary = x*cos + rotate_half(x)*sin).
//   silu_mul: out = T(float(T(silu(g))) * float(u)), silu(g) = g / (1 + exp(-g))
//             (engine/qwen.py:49-50).
#include "sdl_common.cuh"

#include <algorithm>

namespace {

constexpr int kNormThreads = 256;

template <typename T>
__global__ void __launch_bounds__(kNormThreads) rmsnorm_kernel(const T* __restrict__ x, int64_t xs,
                                                               const T* __restrict__ delta, int64_t ds,
                                                               T* __restrict__ x_out, int64_t xos,
                                                               const T* __restrict__ w, T* __restrict__ out,
                                                               int64_t os, int dim, float eps) {
    __shared__ float s_red[32];
    const int64_t row = blockIdx.x;
    const T* xr = x + row * xs;
    float ss = 0.f;
    for (int i = threadIdx.x; i < dim; i += kNormThreads) {
        float v = to_f32<T>(xr[i]);
        if (delta != nullptr) {
            const T h = from_f32<T>(__fadd_rn(v, to_f32<T>(delta[row * ds + i])));
            x_out[row * xos + i] = h;
            v = to_f32<T>(h);
        }
        ss = __fmaf_rn(v, v, ss);
    }
    ss = block_sum<float>(ss, s_red);
    // the mean as sum * fl(1/dim), the form of a mean reduction's final scale
    const float r = __fsqrt_rn(__fadd_rn(__fmul_rn(ss, __frcp_rn((float)dim)), eps));
    const T* hr = delta != nullptr ? x_out + row * xos : xr;
    for (int i = threadIdx.x; i < dim; i += kNormThreads) {
        const float v = to_f32<T>(hr[i]);
        out[row * os + i] = from_f32<T>(__fmul_rn(__fdiv_rn(v, r), to_f32<T>(w[i])));
    }
}

// rmsnorm_kernel with the row held in registers (K elements per thread,
// dim <= K * kNormThreads): every load of x, delta and the weight is issued
// before the reduction, so a row costs one memory round trip instead of one
// per loop iteration, and the output is written from registers.  Same
// operations in the same order per element and per thread, so the results
// are bit-identical to rmsnorm_kernel's.
template <typename T, int K>
__global__ void __launch_bounds__(kNormThreads) rmsnorm_regs_kernel(const T* __restrict__ x, int64_t xs,
                                                                    const T* __restrict__ delta, int64_t ds,
                                                                    T* __restrict__ x_out, int64_t xos,
                                                                    const T* __restrict__ w, T* __restrict__ out,
                                                                    int64_t os, int dim, float eps) {
    __shared__ float s_red[32];
    const int64_t row = blockIdx.x;
    T xv[K], dv[K], wv[K];
#pragma unroll
    for (int k = 0; k < K; ++k) {
        const int i = threadIdx.x + k * kNormThreads;
        if (i < dim) {
            xv[k] = x[row * xs + i];
            if (delta != nullptr) dv[k] = delta[row * ds + i];
            wv[k] = w[i];
        }
    }
    float v[K];
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < K; ++k) {
        const int i = threadIdx.x + k * kNormThreads;
        v[k] = 0.f;
        if (i < dim) {
            v[k] = to_f32<T>(xv[k]);
            if (delta != nullptr) {
                const T h = from_f32<T>(__fadd_rn(v[k], to_f32<T>(dv[k])));
                x_out[row * xos + i] = h;
                v[k] = to_f32<T>(h);
            }
            ss = __fmaf_rn(v[k], v[k], ss);
        }
    }
    ss = block_sum<float>(ss, s_red);
    const float r = __fsqrt_rn(__fadd_rn(__fmul_rn(ss, __frcp_rn((float)dim)), eps));
#pragma unroll
    for (int k = 0; k < K; ++k) {
        const int i = threadIdx.x + k * kNormThreads;
        if (i < dim) out[row * os + i] = from_f32<T>(__fmul_rn(__fdiv_rn(v[k], r), to_f32<T>(wv[k])));
    }
}

// rmsnorm_kernel over rows held as 16-byte pieces: one CTA per row, one
// 8-element piece per thread (dim % 8 == 0, dim <= 8 * 1024, 16-byte aligned
// rows), so a row costs one 16-byte load per input per thread.  The sum of
// squares is per-thread in element order, then a warp tree, then the warps'
// sums in order: another fixed order than rmsnorm_kernel's.
template <typename T>
__global__ void __launch_bounds__(1024) rmsnorm_vec_kernel(const T* __restrict__ x, int64_t xs,
                                                           const T* __restrict__ delta, int64_t ds,
                                                           T* __restrict__ x_out, int64_t xos,
                                                           const T* __restrict__ w, T* __restrict__ out,
                                                           int64_t os, int dim, float eps) {
    __shared__ float s_warp[32];
    __shared__ float s_total;
    const int64_t row = blockIdx.x;
    const int c = threadIdx.x * 8;
    const bool on = c < dim;
    float v[8];
    uint4 wv = make_uint4(0, 0, 0, 0);
    float ss = 0.f;
    if (on) {
        const uint4 xv = *reinterpret_cast<const uint4*>(x + row * xs + c);
        wv = *reinterpret_cast<const uint4*>(w + c);
        const T* xe = reinterpret_cast<const T*>(&xv);
        if (delta != nullptr) {
            const uint4 dv = *reinterpret_cast<const uint4*>(delta + row * ds + c);
            const T* de = reinterpret_cast<const T*>(&dv);
            uint4 hv;
            T* he = reinterpret_cast<T*>(&hv);
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                he[k] = from_f32<T>(__fadd_rn(to_f32<T>(xe[k]), to_f32<T>(de[k])));
                v[k] = to_f32<T>(he[k]);
            }
            *reinterpret_cast<uint4*>(x_out + row * xos + c) = hv;
        } else {
#pragma unroll
            for (int k = 0; k < 8; ++k) v[k] = to_f32<T>(xe[k]);
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) ss = __fmaf_rn(v[k], v[k], ss);
    }
    ss = warp_sum(ss);
    const int warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
    if ((threadIdx.x & 31) == 0) s_warp[warp] = ss;
    __syncthreads();
    if (threadIdx.x == 0) {
        float t = 0.f;
        for (int i = 0; i < nw; ++i) t = __fadd_rn(t, s_warp[i]);
        s_total = t;
    }
    __syncthreads();
    if (!on) return;
    const float r = __fsqrt_rn(__fadd_rn(__fmul_rn(s_total, __frcp_rn((float)dim)), eps));
    const T* we = reinterpret_cast<const T*>(&wv);
    uint4 ov;
    T* oe = reinterpret_cast<T*>(&ov);
#pragma unroll
    for (int k = 0; k < 8; ++k) oe[k] = from_f32<T>(__fmul_rn(__fdiv_rn(v[k], r), to_f32<T>(we[k])));
    *reinterpret_cast<uint4*>(out + row * os + c) = ov;
}

// One thread per (row, head, i < d/2) pair of rotated elements.
template <typename T>
__global__ void rope_kernel(T* __restrict__ x, int64_t xs, int heads, int d, const T* __restrict__ cs,
                            int64_t cs_stride, const T* __restrict__ sn, int64_t sn_stride, int rows) {
    const int half = d / 2;
    const int per_row = heads * half;  // the host keeps rows * per_row below 2^31: 32-bit index math
    const int n = rows * per_row;
    for (int t = blockIdx.x * blockDim.x + threadIdx.x; t < n; t += gridDim.x * blockDim.x) {
        const int r = t / per_row;
        const int rem = t - r * per_row;
        const int h = rem / half;
        const int i = rem - h * half;
        T* p = x + (int64_t)r * xs + (int64_t)h * d;
        const float x1 = to_f32<T>(p[i]), x2 = to_f32<T>(p[i + half]);
        const T* c = cs + r * cs_stride;
        const T* s = sn + r * sn_stride;
        const float c1 = to_f32<T>(c[i]), c2 = to_f32<T>(c[i + half]);
        const float s1 = to_f32<T>(s[i]), s2 = to_f32<T>(s[i + half]);
        // rotate_half(x) = (-x2, x1): each product and the sum round to T
        const float a1 = round_trip<T>(__fmul_rn(x1, c1)), b1 = round_trip<T>(__fmul_rn(-x2, s1));
        const float a2 = round_trip<T>(__fmul_rn(x2, c2)), b2 = round_trip<T>(__fmul_rn(x1, s2));
        p[i] = from_f32<T>(__fadd_rn(a1, b1));
        p[i + half] = from_f32<T>(__fadd_rn(a2, b2));
    }
}

template <typename T>
__global__ void silu_mul_kernel(const T* __restrict__ g, const T* __restrict__ u, T* __restrict__ out, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const float gv = to_f32<T>(g[i]);
        const float sv = round_trip<T>(__fdiv_rn(gv, __fadd_rn(1.f, expf(-gv))));
        out[i] = from_f32<T>(__fmul_rn(sv, to_f32<T>(u[i])));
    }
}

// SwiGLU gate over fused rows [gate | up]: one thread per (row, i).
template <typename T>
__global__ void swiglu_kernel(const T* __restrict__ x, int64_t xs, T* __restrict__ out, int64_t os, int rows,
                              int inter) {
    const int64_t n = (int64_t)rows * inter;
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < n; t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = t / inter;
        const int i = (int)(t - r * inter);
        const T* xr = x + r * xs;
        const float gv = to_f32<T>(xr[i]);
        const float sv = round_trip<T>(__fdiv_rn(gv, __fadd_rn(1.f, expf(-gv))));
        out[r * os + i] = from_f32<T>(__fmul_rn(sv, to_f32<T>(xr[inter + i])));
    }
}

// The same on pairs of columns: one row per blockIdx.y, 4-byte accesses
// (even inter and row strides, 4-byte aligned rows).
template <typename T> struct Pair2;
template <> struct Pair2<__nv_bfloat16> { using type = __nv_bfloat162; };
template <> struct Pair2<__half> { using type = __half2; };

template <typename T>
__global__ void swiglu_pair_kernel(const T* __restrict__ x, int64_t xs, T* __restrict__ out, int64_t os, int inter) {
    using T2 = typename Pair2<T>::type;
    const int i = 2 * (blockIdx.x * blockDim.x + threadIdx.x);
    if (i >= inter) return;
    const T* xr = x + (int64_t)blockIdx.y * xs;
    const T2 g = *reinterpret_cast<const T2*>(xr + i);
    const T2 u = *reinterpret_cast<const T2*>(xr + inter + i);
    const float g0 = to_f32<T>(g.x), g1 = to_f32<T>(g.y);
    const float s0 = round_trip<T>(__fdiv_rn(g0, __fadd_rn(1.f, expf(-g0))));
    const float s1 = round_trip<T>(__fdiv_rn(g1, __fadd_rn(1.f, expf(-g1))));
    T2 y;
    y.x = from_f32<T>(__fmul_rn(s0, to_f32<T>(u.x)));
    y.y = from_f32<T>(__fmul_rn(s1, to_f32<T>(u.y)));
    *reinterpret_cast<T2*>(out + (int64_t)blockIdx.y * os + i) = y;
}

// The same on 8 columns per thread (16-byte accesses: inter and the row
// strides multiples of 8, 16-byte aligned rows); one row per blockIdx.y.
template <typename T>
__global__ void __launch_bounds__(128) swiglu_vec_kernel(const T* __restrict__ x, int64_t xs, T* __restrict__ out,
                                                         int64_t os, int inter) {
    const int i = 8 * (blockIdx.x * blockDim.x + threadIdx.x);
    if (i >= inter) return;
    const T* xr = x + (int64_t)blockIdx.y * xs;
    const uint4 gv = *reinterpret_cast<const uint4*>(xr + i);
    const uint4 uv = *reinterpret_cast<const uint4*>(xr + inter + i);
    const T* ge = reinterpret_cast<const T*>(&gv);
    const T* ue = reinterpret_cast<const T*>(&uv);
    uint4 yv;
    T* ye = reinterpret_cast<T*>(&yv);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const float g = to_f32<T>(ge[k]);
        const float sv = round_trip<T>(__fdiv_rn(g, __fadd_rn(1.f, expf(-g))));
        ye[k] = from_f32<T>(__fmul_rn(sv, to_f32<T>(ue[k])));
    }
    *reinterpret_cast<uint4*>(out + (int64_t)blockIdx.y * os + i) = yv;
}

int grid_for(int64_t n, int threads) {
    const int64_t b = (n + threads - 1) / threads;
    return (int)std::min<int64_t>(std::max<int64_t>(b, 1), 148 * 16);
}

// Rows of up to 16 * kNormThreads elements take the register-held kernel.
template <typename T>
void launch_rmsnorm(const void* x, int64_t xs, const void* delta, int64_t ds, void* x_out, int64_t xos,
                    const void* weight, void* out, int64_t os, int rows, int dim, float eps, cudaStream_t st) {
    const T* xp = static_cast<const T*>(x);
    const T* dp = static_cast<const T*>(delta);
    T* xo = static_cast<T*>(x_out);
    const T* wp = static_cast<const T*>(weight);
    T* op = static_cast<T*>(out);
    auto al16 = [](const void* q) { return reinterpret_cast<uintptr_t>(q) % 16 == 0; };
    if (dim % 8 == 0 && dim <= 8 * 1024 && xs % 8 == 0 && os % 8 == 0 && al16(x) && al16(weight) && al16(out) &&
        (delta == nullptr || (ds % 8 == 0 && xos % 8 == 0 && al16(delta) && al16(x_out)))) {
        const int threads = (dim / 8 + 31) / 32 * 32;
        rmsnorm_vec_kernel<T><<<rows, threads, 0, st>>>(xp, xs, dp, ds, xo, xos, wp, op, os, dim, eps);
    } else if (dim <= 4 * kNormThreads)
        rmsnorm_regs_kernel<T, 4><<<rows, kNormThreads, 0, st>>>(xp, xs, dp, ds, xo, xos, wp, op, os, dim, eps);
    else if (dim <= 8 * kNormThreads)
        rmsnorm_regs_kernel<T, 8><<<rows, kNormThreads, 0, st>>>(xp, xs, dp, ds, xo, xos, wp, op, os, dim, eps);
    else if (dim <= 16 * kNormThreads)
        rmsnorm_regs_kernel<T, 16><<<rows, kNormThreads, 0, st>>>(xp, xs, dp, ds, xo, xos, wp, op, os, dim, eps);
    else
        rmsnorm_kernel<T><<<rows, kNormThreads, 0, st>>>(xp, xs, dp, ds, xo, xos, wp, op, os, dim, eps);
}

}  // namespace

extern "C" int sdl_rmsnorm(const void* x, int64_t x_stride, const void* delta, int64_t delta_stride, void* x_out,
                           int64_t x_out_stride, const void* weight, void* out, int64_t out_stride, int32_t rows,
                           int32_t dim, float eps, int32_t dtype, void* stream) {
    if (!x || !weight || !out || rows < 0 || dim < 1 || (delta && !x_out))
        return sdl::fail(SDL_ERR_INVALID, "sdl_rmsnorm: bad arguments");
    if (rows == 0) return SDL_OK;
    if (dtype != SDL_BF16 && dtype != SDL_F16) return sdl::fail(SDL_ERR_UNSUPPORTED, "sdl_rmsnorm: 16-bit dtypes only");
    cudaStream_t st = sdl::as_stream(stream);
    if (dtype == SDL_BF16) launch_rmsnorm<__nv_bfloat16>(x, x_stride, delta, delta_stride, x_out, x_out_stride, weight,
                                                         out, out_stride, rows, dim, eps, st);
    else launch_rmsnorm<__half>(x, x_stride, delta, delta_stride, x_out, x_out_stride, weight, out, out_stride, rows,
                                dim, eps, st);
    return sdl::check_launch("rmsnorm_kernel");
}

extern "C" int sdl_rope(void* x, int64_t x_row_stride, int32_t rows, int32_t heads, int32_t head_dim,
                        const void* cos, int64_t cos_row_stride, const void* sin, int64_t sin_row_stride,
                        int32_t dtype, void* stream) {
    if (!x || !cos || !sin || rows < 0 || heads < 1 || head_dim < 2 || head_dim % 2)
        return sdl::fail(SDL_ERR_INVALID, "sdl_rope: bad arguments");
    if ((int64_t)rows * heads * (head_dim / 2) >= (int64_t(1) << 31))
        return sdl::fail(SDL_ERR_UNSUPPORTED, "sdl_rope: more than 2^31 rotated pairs in one call");
    if (rows == 0) return SDL_OK;
    cudaStream_t st = sdl::as_stream(stream);
    const int64_t n = (int64_t)rows * heads * (head_dim / 2);
    const int grid = grid_for(n, 256);
    if (dtype == SDL_BF16) {
        using T = __nv_bfloat16;
        rope_kernel<T><<<grid, 256, 0, st>>>((T*)x, x_row_stride, heads, head_dim, (const T*)cos, cos_row_stride,
                                              (const T*)sin, sin_row_stride, rows);
    } else if (dtype == SDL_F16) {
        using T = __half;
        rope_kernel<T><<<grid, 256, 0, st>>>((T*)x, x_row_stride, heads, head_dim, (const T*)cos, cos_row_stride,
                                              (const T*)sin, sin_row_stride, rows);
    } else {
        return sdl::fail(SDL_ERR_UNSUPPORTED, "sdl_rope: 16-bit dtypes only");
    }
    return sdl::check_launch("rope_kernel");
}

extern "C" int sdl_silu_mul(const void* gate, const void* up, void* out, int64_t n, int32_t dtype, void* stream) {
    if (!gate || !up || !out || n < 0) return sdl::fail(SDL_ERR_INVALID, "sdl_silu_mul: bad arguments");
    if (n == 0) return SDL_OK;
    cudaStream_t st = sdl::as_stream(stream);
    const int grid = grid_for(n, 256);
    if (dtype == SDL_BF16) {
        using T = __nv_bfloat16;
        silu_mul_kernel<T><<<grid, 256, 0, st>>>((const T*)gate, (const T*)up, (T*)out, n);
    } else if (dtype == SDL_F16) {
        using T = __half;
        silu_mul_kernel<T><<<grid, 256, 0, st>>>((const T*)gate, (const T*)up, (T*)out, n);
    } else {
        return sdl::fail(SDL_ERR_UNSUPPORTED, "sdl_silu_mul: 16-bit dtypes only");
    }
    return sdl::check_launch("silu_mul_kernel");
}

extern "C" int sdl_swiglu(const void* x, int64_t x_row_stride, void* out, int64_t out_row_stride, int32_t rows,
                          int32_t inter, int32_t dtype, void* stream) {
    if (!x || !out || rows < 0 || inter < 1 || x_row_stride < 2 * (int64_t)inter || out_row_stride < inter)
        return sdl::fail(SDL_ERR_INVALID, "sdl_swiglu: bad arguments");
    if (rows == 0) return SDL_OK;
    cudaStream_t st = sdl::as_stream(stream);
    auto al4 = [](const void* q) { return reinterpret_cast<uintptr_t>(q) % 4 == 0; };
    auto al16 = [](const void* q) { return reinterpret_cast<uintptr_t>(q) % 16 == 0; };
    if (inter % 8 == 0 && x_row_stride % 8 == 0 && out_row_stride % 8 == 0 && al16(x) && al16(out) && rows <= 65535 &&
        (dtype == SDL_BF16 || dtype == SDL_F16)) {
        const dim3 grid((inter / 8 + 127) / 128, rows);
        if (dtype == SDL_BF16) {
            using T = __nv_bfloat16;
            swiglu_vec_kernel<T><<<grid, 128, 0, st>>>((const T*)x, x_row_stride, (T*)out, out_row_stride, inter);
        } else {
            using T = __half;
            swiglu_vec_kernel<T><<<grid, 128, 0, st>>>((const T*)x, x_row_stride, (T*)out, out_row_stride, inter);
        }
        return sdl::check_launch("swiglu_vec_kernel");
    }
    if (inter % 2 == 0 && x_row_stride % 2 == 0 && out_row_stride % 2 == 0 && al4(x) && al4(out) && rows <= 65535 &&
        (dtype == SDL_BF16 || dtype == SDL_F16)) {
        const dim3 grid((inter / 2 + 255) / 256, rows);
        if (dtype == SDL_BF16) {
            using T = __nv_bfloat16;
            swiglu_pair_kernel<T><<<grid, 256, 0, st>>>((const T*)x, x_row_stride, (T*)out, out_row_stride, inter);
        } else {
            using T = __half;
            swiglu_pair_kernel<T><<<grid, 256, 0, st>>>((const T*)x, x_row_stride, (T*)out, out_row_stride, inter);
        }
        return sdl::check_launch("swiglu_pair_kernel");
    }
    const int grid = grid_for((int64_t)rows * inter, 256);
    if (dtype == SDL_BF16) {
        using T = __nv_bfloat16;
        swiglu_kernel<T><<<grid, 256, 0, st>>>((const T*)x, x_row_stride, (T*)out, out_row_stride, rows, inter);
    } else if (dtype == SDL_F16) {
        using T = __half;
        swiglu_kernel<T><<<grid, 256, 0, st>>>((const T*)x, x_row_stride, (T*)out, out_row_stride, rows, inter);
    } else {
        return sdl::fail(SDL_ERR_UNSUPPORTED, "sdl_swiglu: 16-bit dtypes only");
    }
    return sdl::check_launch("swiglu_kernel");
}
