// Sampling kernels: temperature softmax / greedy one-hot, first-index argmax,
// the exact integer inverse-CDF draw, and the fused rejection sampler of a
// speculative round.
//
// The inverse-CDF rule is defined on exact integers so that the kernel and
// any CPU restatement agree bit-for-bit regardless of summation order:
//   W_i = floor(w_i * 2^62)  (w_i fp32 in [0, 4); NaN / negatives count as 0)
//   S   = sum_i W_i          (exact in uint64)
//   U   = floor(u * 2^64)    (u fp32 uniform in [0, 1))
//   target = floor(U * S / 2^64)
//   token  = min{ i : W_0 + ... + W_i > target }
// It replaces torch.multinomial(probs, 1) in sample_token
// (specdec/sampler.py:59-69) and PagedScheduler._sample
// (engine/scheduler.py:235-239) given the same pre-drawn uniforms.
#include "sdl_common.cuh"

namespace {

constexpr double kTwo62 = 4611686018427387904.0;
constexpr double kTwo64 = 18446744073709551616.0;

// floor(w * 2^62): the fp32 product with a power of two is exact (no
// rounding below 2^66), and the truncating conversion to u64 saturates
// (w >= 4 gives 2^64 - 1) and maps NaN and w <= 0 to 0.
SDL_DEV uint64_t wfix(float w) { return __float2ull_rz(__fmul_rn(w, 4611686018427387904.0f)); }

SDL_DEV uint64_t ufix(float u) {
    if (!(u > 0.f)) return 0ull;
    double x = (double)u * kTwo64;
    if (x >= kTwo64) return 0xffffffffffffffffull;
    return __double2ull_rz(x);
}

SDL_DEV uint64_t warp_sum_u64(uint64_t v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

SDL_DEV uint64_t warp_incl_scan_u64(uint64_t v, int lane) {
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        uint64_t y = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += y;
    }
    return v;
}

// Block-wide draw with the rule above.  Warp w owns a contiguous range of the
// row; lanes read it coalesced.  `wf(i)` returns the fp32 weight of index i.
// Returns the index to thread 0 via the return value of every thread; -1 when
// the weights sum to zero.  Needs blockDim == 1024.
template <typename WF>
SDL_DEV int block_draw(WF wf, int V, float u, uint64_t* s_wsum /*[32]*/, int* s_tok) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    int wseg = (V + nw - 1) / nw;
    wseg = (wseg + 31) & ~31;
    const int lo = warp * wseg, hi = min(V, lo + wseg);
    uint64_t s = 0;
    for (int i = lo + lane; i < hi; i += 32) s += wfix(wf(i));
    s = warp_sum_u64(s);
    if (lane == 0) s_wsum[warp] = s;
    if (threadIdx.x == 0) *s_tok = -1;
    __syncthreads();
    uint64_t excl = 0, S = 0;
    for (int w = 0; w < nw; ++w) {
        if (w < warp) excl += s_wsum[w];
        S += s_wsum[w];
    }
    if (S != 0) {
        const uint64_t target = __umul64hi(ufix(u), S);
        if (excl <= target && target < excl + s_wsum[warp]) {
            uint64_t run = excl;
            for (int base = lo; base < hi; base += 32) {
                const int i = base + lane;
                const uint64_t val = i < hi ? wfix(wf(i)) : 0ull;
                const uint64_t pre = warp_incl_scan_u64(val, lane);
                const unsigned hit = __ballot_sync(0xffffffffu, run + pre > target);
                if (hit) {
                    if (lane == 0) *s_tok = base + __ffs(hit) - 1;
                    break;
                }
                run += __shfl_sync(0xffffffffu, pre, 31);
            }
        }
    }
    __syncthreads();
    return *s_tok;
}

// Block argmax, first index on ties.
template <typename T>
SDL_DEV int block_argmax(const T* x, int V, float* s_val, int* s_idx) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    float best = -INFINITY;
    int bi = 0x7fffffff;
    for (int i = threadIdx.x; i < V; i += blockDim.x) {
        const float v = to_f32<T>(x[i]);
        if (v > best || (v == best && i < bi)) { best = v; bi = i; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
    }
    if (lane == 0) { s_val[warp] = best; s_idx[warp] = bi; }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < nw; ++w)
            if (s_val[w] > s_val[0] || (s_val[w] == s_val[0] && s_idx[w] < s_idx[0])) {
                s_val[0] = s_val[w];
                s_idx[0] = s_idx[w];
            }
        if (s_idx[0] == 0x7fffffff) s_idx[0] = 0;  // all -inf / NaN: row 0 like an empty argmax
    }
    __syncthreads();
    const int r = s_idx[0];
    __syncthreads();
    return r;
}

template <typename T>
__global__ void __launch_bounds__(1024) probs_kernel(const T* __restrict__ logits, int64_t row_stride, int V, float temp,
                                                     int greedy, float* __restrict__ out, int64_t out_stride) {
    __shared__ float s_val[32];
    __shared__ int s_idx[32];
    const T* x = logits + blockIdx.x * row_stride;
    float* o = out + blockIdx.x * out_stride;
    if (greedy) {
        const int am = block_argmax<T>(x, V, s_val, s_idx);
        for (int i = threadIdx.x; i < V; i += blockDim.x) o[i] = i == am ? 1.f : 0.f;
        return;
    }
    float m = -INFINITY;
    for (int i = threadIdx.x; i < V; i += blockDim.x) m = fmaxf(m, to_f32<T>(x[i]) / temp);
    m = warp_max(m);
    if ((threadIdx.x & 31) == 0) s_val[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x < 32) {
        float v = threadIdx.x < (blockDim.x >> 5) ? s_val[threadIdx.x] : -INFINITY;
        v = warp_max(v);
        if (threadIdx.x == 0) s_val[0] = v;
    }
    __syncthreads();
    m = s_val[0];
    __syncthreads();
    float sum = 0.f;
    for (int i = threadIdx.x; i < V; i += blockDim.x) {
        const float e = expf(to_f32<T>(x[i]) / temp - m);
        o[i] = e;
        sum += e;
    }
    sum = warp_sum(sum);
    if ((threadIdx.x & 31) == 0) s_val[threadIdx.x >> 5] = sum;
    __syncthreads();
    if (threadIdx.x < 32) {
        float v = threadIdx.x < (blockDim.x >> 5) ? s_val[threadIdx.x] : 0.f;
        v = warp_sum(v);
        if (threadIdx.x == 0) s_val[0] = v;
    }
    __syncthreads();
    const float z = s_val[0];
    for (int i = threadIdx.x; i < V; i += blockDim.x) o[i] = o[i] / z;
}

template <typename T>
__global__ void __launch_bounds__(1024) argmax_kernel(const T* __restrict__ logits, int64_t row_stride, int V,
                                                      int* __restrict__ out) {
    __shared__ float s_val[32];
    __shared__ int s_idx[32];
    const int am = block_argmax<T>(logits + blockIdx.x * row_stride, V, s_val, s_idx);
    if (threadIdx.x == 0) out[blockIdx.x] = am;
}

__global__ void __launch_bounds__(1024) sample_kernel(const float* __restrict__ w, int64_t row_stride, int V,
                                                      const float* __restrict__ uniforms, int64_t nu,
                                                      const int64_t* u_base, int64_t u_off, int* out, int* err) {
    __shared__ uint64_t s_wsum[32];
    __shared__ int s_tok;
    const int64_t ui = (u_base ? *u_base : 0) + u_off + blockIdx.x;
    if (ui < 0 || ui >= nu) {
        if (threadIdx.x == 0) { sdl_raise(err, SDL_DEVERR_UNIFORMS); out[blockIdx.x] = 0; }
        return;
    }
    const float u = uniforms[ui];
    const float* x = w + blockIdx.x * row_stride;
    const int tok = block_draw([&](int i) { return x[i]; }, V, u, s_wsum, &s_tok);
    if (threadIdx.x == 0) {
        if (tok < 0) { sdl_raise(err, SDL_DEVERR_BAD_SAMPLE); out[blockIdx.x] = 0; }
        else out[blockIdx.x] = tok;
    }
}

__global__ void counter_add_kernel(int64_t* c, int64_t d) { *c += d; }

// Phase A + B of the rejection sampler (one CTA): acceptance probabilities in
// fp64 (specdec/sampler.py:86-92), then the sequential walk that decides how
// many uniforms each sequence consumes (engine/spec_scheduler.py:67-87).
__global__ void __launch_bounds__(1024) spec_accept_kernel(
    const float* __restrict__ p, int64_t p_sb, int64_t p_sj, const float* __restrict__ q, int64_t q_sb, int64_t q_sj,
    const int* __restrict__ p_arg, const int* __restrict__ prop, int B, int gamma, int greedy,
    const float* __restrict__ uniforms, int64_t nu, int64_t* u_base, int64_t u_skip, int* tokens, int* n_out,
    int* n_acc, int* u_final_bits, int* err) {
    extern __shared__ double s_dyn[];
    double* a = s_dyn;                                                  // [B*gamma]
    float* uc = reinterpret_cast<float*>(s_dyn + (size_t)B * gamma);    // [B*(gamma+1)]
    const int64_t base = (u_base ? *u_base : 0) + u_skip;
    for (int idx = threadIdx.x; idx < B * gamma; idx += blockDim.x) {
        const int b = idx / gamma, j = idx % gamma;
        const int x = prop[idx];
        double acc;
        if (greedy) {
            acc = p_arg[b * (gamma + 1) + j] == x ? 1.0 : 0.0;
        } else {
            const double pv = p[b * p_sb + j * p_sj + x];
            const double qv = q[b * q_sb + j * q_sj + x];
            if (qv <= 1e-12) acc = pv > 1e-12 ? 1.0 : 0.0;
            else acc = fmin(1.0, pv / qv);
        }
        a[idx] = acc;
    }
    for (int i = threadIdx.x; i < B * (gamma + 1); i += blockDim.x) {
        const int64_t ui = base + i;
        uc[i] = (uniforms && ui >= 0 && ui < nu) ? uniforms[ui] : __int_as_float(0x7fc00000);
    }
    __syncthreads();
    if (threadIdx.x >= 32) return;
    const int lane = threadIdx.x;
    int off = 0;
    bool bad_u = false;
    for (int b = 0; b < B; ++b) {
        bool reject = false;
        if (lane < gamma) {
            const float u = uc[off + lane];
            if (uniforms && u != u) bad_u = true;
            reject = !((double)(uniforms ? u : 0.f) < a[b * gamma + lane]);
        }
        const unsigned rj = __ballot_sync(0xffffffffu, reject);
        const int r = rj ? __ffs(rj) - 1 : gamma;
        const int consumed = r < gamma ? r + 2 : gamma + 1;
        if (lane == 0) {
            n_acc[b] = r;
            const float uf = uc[off + consumed - 1];
            if (uniforms && uf != uf) bad_u = true;
            u_final_bits[b] = __float_as_int(uf);
            if (greedy) {
                for (int j = 0; j < r; ++j) tokens[b * (gamma + 1) + j] = prop[b * gamma + j];
                tokens[b * (gamma + 1) + r] = p_arg[b * (gamma + 1) + r];
                n_out[b] = r + 1;
            }
        }
        off += consumed;
    }
    bad_u = __any_sync(0xffffffffu, bad_u);
    if (lane == 0) {
        if (bad_u) sdl_raise(err, SDL_DEVERR_UNIFORMS);
        if (u_base) *u_base = base + off;
    }
}

// Phase C (one CTA per sequence): residual or bonus draw over the vocabulary.
__global__ void __launch_bounds__(1024) spec_resample_kernel(const float* __restrict__ p, int64_t p_sb, int64_t p_sj,
                                                             const float* __restrict__ q, int64_t q_sb, int64_t q_sj,
                                                             const int* __restrict__ prop, int gamma, int V,
                                                             const int* n_acc, const int* u_final_bits, int* tokens,
                                                             int* n_out, int* err) {
    __shared__ uint64_t s_wsum[32];
    __shared__ int s_tok;
    const int b = blockIdx.x;
    const int r = n_acc[b];
    const float u = __int_as_float(u_final_bits[b]);
    const float* pr = p + b * p_sb + (int64_t)r * p_sj;
    int tok;
    if (r < gamma) {
        const float* qr = q + b * q_sb + (int64_t)r * q_sj;
        // Residual (p - q)+; fall back to p when its mass is <= 1e-12.
        uint64_t s = 0;
        for (int i = threadIdx.x; i < V; i += blockDim.x) s += wfix(fmaxf(pr[i] - qr[i], 0.f));
        s = warp_sum_u64(s);
        if ((threadIdx.x & 31) == 0) s_wsum[threadIdx.x >> 5] = s;
        __syncthreads();
        uint64_t S = 0;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) S += s_wsum[w];
        __syncthreads();
        if ((double)S / kTwo62 <= 1e-12) tok = block_draw([&](int i) { return pr[i]; }, V, u, s_wsum, &s_tok);
        else tok = block_draw([&](int i) { return fmaxf(pr[i] - qr[i], 0.f); }, V, u, s_wsum, &s_tok);
    } else {
        tok = block_draw([&](int i) { return pr[i]; }, V, u, s_wsum, &s_tok);
    }
    if (threadIdx.x == 0) {
        if (tok < 0) { sdl_raise(err, SDL_DEVERR_BAD_SAMPLE); tok = 0; }
        for (int j = 0; j < r; ++j) tokens[b * (gamma + 1) + j] = prop[b * gamma + j];
        tokens[b * (gamma + 1) + r] = tok;
        n_out[b] = r + 1;
    }
}

}  // namespace

// Canonical temperature softmax (csrc/sampler_logits.cu).
int sdl_probs_canon(const void* logits, int32_t dtype, int64_t row_stride, int32_t rows, int32_t vocab, float temp,
                    float* probs, int64_t probs_stride, cudaStream_t st);

extern "C" int sdl_logits_to_probs(const void* logits, int32_t dtype, int64_t row_stride, int32_t rows, int32_t vocab,
                                   float temperature, float eps, int32_t greedy, float* probs, int64_t probs_stride,
                                   void* stream) {
    if (!logits || !probs || rows < 0 || vocab < 1 || row_stride < vocab || probs_stride < vocab)
        return sdl::fail(SDL_ERR_INVALID, "sdl_logits_to_probs: bad args");
    if (rows == 0) return SDL_OK;
    const float t = temperature > eps ? temperature : eps;
    cudaStream_t st = sdl::as_stream(stream);
    if (!greedy) return sdl_probs_canon(logits, dtype, row_stride, rows, vocab, t, probs, probs_stride, st);
    if (dtype == SDL_F32)
        probs_kernel<float><<<rows, 1024, 0, st>>>((const float*)logits, row_stride, vocab, t, greedy, probs, probs_stride);
    else if (dtype == SDL_BF16)
        probs_kernel<__nv_bfloat16><<<rows, 1024, 0, st>>>((const __nv_bfloat16*)logits, row_stride, vocab, t, greedy,
                                                           probs, probs_stride);
    else if (dtype == SDL_F16)
        probs_kernel<__half><<<rows, 1024, 0, st>>>((const __half*)logits, row_stride, vocab, t, greedy, probs,
                                                    probs_stride);
    else
        return sdl::fail(SDL_ERR_UNSUPPORTED, "sdl_logits_to_probs: dtype");
    return sdl::check_launch("probs_kernel");
}

extern "C" int sdl_argmax_rows(const void* logits, int32_t dtype, int64_t row_stride, int32_t rows, int32_t vocab,
                               int32_t* out, void* stream) {
    if (!logits || !out || rows < 0 || vocab < 1 || row_stride < vocab)
        return sdl::fail(SDL_ERR_INVALID, "sdl_argmax_rows: bad args");
    if (rows == 0) return SDL_OK;
    cudaStream_t st = sdl::as_stream(stream);
    if (dtype == SDL_F32) argmax_kernel<float><<<rows, 1024, 0, st>>>((const float*)logits, row_stride, vocab, out);
    else if (dtype == SDL_BF16)
        argmax_kernel<__nv_bfloat16><<<rows, 1024, 0, st>>>((const __nv_bfloat16*)logits, row_stride, vocab, out);
    else if (dtype == SDL_F16) argmax_kernel<__half><<<rows, 1024, 0, st>>>((const __half*)logits, row_stride, vocab, out);
    else return sdl::fail(SDL_ERR_UNSUPPORTED, "sdl_argmax_rows: dtype");
    return sdl::check_launch("argmax_kernel");
}

extern "C" int sdl_sample_rows(const float* weights, int64_t row_stride, int32_t rows, int32_t vocab,
                               const float* uniforms, int64_t num_uniforms, const int64_t* u_base, int64_t u_offset,
                               int32_t* out, int32_t* err, void* stream) {
    if (!weights || !uniforms || !out || rows < 0 || vocab < 1 || row_stride < vocab)
        return sdl::fail(SDL_ERR_INVALID, "sdl_sample_rows: bad args");
    if (rows == 0) return SDL_OK;
    sample_kernel<<<rows, 1024, 0, sdl::as_stream(stream)>>>(weights, row_stride, vocab, uniforms, num_uniforms, u_base,
                                                           u_offset, out, err);
    return sdl::check_launch("sample_kernel");
}

extern "C" int sdl_counter_add(int64_t* counter, int64_t delta, void* stream) {
    if (!counter) return sdl::fail(SDL_ERR_INVALID, "sdl_counter_add: NULL counter");
    counter_add_kernel<<<1, 1, 0, sdl::as_stream(stream)>>>(counter, delta);
    return sdl::check_launch("counter_add_kernel");
}

extern "C" size_t sdl_spec_sample_scratch_bytes(int32_t B) { return (size_t)(B > 0 ? B : 0) * 2 * sizeof(int32_t); }

extern "C" int sdl_spec_sample(const float* p, int64_t p_sb, int64_t p_sj, const float* q, int64_t q_sb, int64_t q_sj,
                               const int32_t* p_arg, const int32_t* proposals, int32_t B, int32_t gamma, int32_t vocab,
                               int32_t greedy, const float* uniforms, int64_t num_uniforms, int64_t* u_base,
                               int64_t u_skip, int32_t* tokens, int32_t* n_out, int32_t* scratch_i32, int32_t* err,
                               void* stream) {
    if (B < 0 || gamma < 1 || gamma > 32 || vocab < 1 || !proposals || !tokens || !n_out || !scratch_i32)
        return sdl::fail(SDL_ERR_INVALID, "sdl_spec_sample: bad args (gamma must be 1..32)");
    if (greedy && !p_arg) return sdl::fail(SDL_ERR_INVALID, "sdl_spec_sample: greedy mode needs p_arg");
    if (!greedy && (!p || !q || !uniforms))
        return sdl::fail(SDL_ERR_INVALID, "sdl_spec_sample: sampling mode needs p, q and uniforms");
    if (B == 0) return SDL_OK;
    const size_t smem = (size_t)B * gamma * sizeof(double) + (size_t)B * (gamma + 1) * sizeof(float);
    if (smem > 200 * 1024) return sdl::fail(SDL_ERR_INVALID, "sdl_spec_sample: batch too large for one accept CTA");
    cudaStream_t st = sdl::as_stream(stream);
    static size_t configured = 0;
    if (smem > 48 * 1024 && smem > configured) {
        cudaError_t e = cudaFuncSetAttribute(spec_accept_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return sdl::fail(SDL_ERR_CUDA, cudaGetErrorString(e));
        configured = smem;
    }
    int32_t* n_acc = scratch_i32;
    int32_t* u_bits = scratch_i32 + B;
    spec_accept_kernel<<<1, 1024, smem, st>>>(p, p_sb, p_sj, q, q_sb, q_sj, p_arg, proposals, B, gamma, greedy,
                                              uniforms, num_uniforms, u_base, u_skip, tokens, n_out, n_acc, u_bits,
                                              err);
    int rc = sdl::check_launch("spec_accept_kernel");
    if (rc != SDL_OK || greedy) return rc;
    spec_resample_kernel<<<B, 1024, 0, st>>>(p, p_sb, p_sj, q, q_sb, q_sj, proposals, gamma, vocab, n_acc, u_bits,
                                             tokens, n_out, err);
    return sdl::check_launch("spec_resample_kernel");
}
