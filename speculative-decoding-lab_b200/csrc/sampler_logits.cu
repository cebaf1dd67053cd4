// Logits-in sampling: canonical chunked softmax statistics, draws straight
// from logits, and the fused rejection sampler of a speculative round that
// never materialises a probability row.
//
// Canonical softmax.  p = softmax(logits / T) in fp32 (specdec/sampler.py:
// 19-36) needs a row maximum m and a row sum s.  The maximum is exact; the
// sum's rounding depends on the summation order, so this file fixes it:
//   * x/T is the correctly rounded quotient (skipped when T == 1: x/1 == x);
//   * the row is cut into chunks of kChunk = 8192 elements;
//   * in a chunk, thread t of a 256-thread group owns elements
//     lo + 4t + j + 1024k (k = 0..7 outer, j = 0..3 inner) and adds
//     expf(x/T - m_c) over them in that order (m_c = the chunk maximum;
//     masked -inf logits add expf(-inf) = +0); lanes combine by an xor
//     butterfly (16, 8, 4, 2, 1) and lane 0's value is kept; warps 0..7 are
//     added in order;
//   * chunks merge in order: m = max m_c, s = fma(s_c, expf(m_c - m), s);
//   * p_i = expf(x_i/T - m) * r with r = 1/s correctly rounded (one product
//     per element instead of a divide; within one ulp of the quotient).
// Every kernel here (one CTA per row or one CTA per chunk) evaluates exactly
// these operations with explicit round-to-nearest intrinsics, so p_i is the
// same bit pattern whichever kernel computes it: sdl_logits_to_probs,
// sdl_sample_logits_rows and sdl_spec_sample_logits agree bit for bit, and
// the draws below equal sdl_sample_rows / sdl_spec_sample applied to
// sdl_logits_to_probs' output.
//
// Draws use the integer inverse-CDF rule of sampler.cu (W_i = floor(w_i *
// 2^62), exact u64 sums), so splitting a row across CTAs cannot change them.
#include "sdl_common.cuh"

#include <map>
#include <mutex>

namespace {

constexpr int kChunk = 8192;   // elements per statistics chunk
constexpr int kGroup = 256;    // threads that reduce one chunk
constexpr int kPerThread = kChunk / kGroup;
constexpr int kMaxChunks = 1024;  // vocab <= 8M
// Draws sum integer weights, which is exact in any order, so they use their
// own finer slices: 2048 elements, 8 per thread of a 256-thread CTA.
constexpr int kDrawChunk = 2048;
constexpr int kDrawPerThread = kDrawChunk / kGroup;
constexpr int kMaxDrawChunks = 1024;  // vocab <= 2M for draws

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

SDL_DEV void group_sync(int id) { asm volatile("bar.sync %0, %1;" :: "r"(id), "r"(kGroup) : "memory"); }

// Logical rows of a [B, J, V] logits tensor with strides (sb, sj).
template <typename T>
struct Rows {
    const T* p;
    int64_t sb, sj;
    int J, n;
    SDL_DEV const T* row(int r) const { return p + (int64_t)(r / J) * sb + (int64_t)(r % J) * sj; }
};

// x / T, correctly rounded; x / 1 == x exactly, so T == 1 skips the divide.
SDL_DEV float scaled(float x, float temp) { return temp == 1.f ? x : __fdiv_rn(x, temp); }

// Four consecutive logits [i, i+4) as fp32 (-inf past hi); one vector load
// when the row is aligned for it.
template <typename T>
SDL_DEV void load4(const T* __restrict__ x, int i, int hi, bool vec, float* o);
template <>
SDL_DEV void load4<float>(const float* __restrict__ x, int i, int hi, bool vec, float* o) {
    if (vec && i + 3 < hi) {
        const float4 v = __ldg(reinterpret_cast<const float4*>(x + i));
        o[0] = v.x; o[1] = v.y; o[2] = v.z; o[3] = v.w;
        return;
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) o[j] = i + j < hi ? x[i + j] : -INFINITY;
}
template <typename H>
SDL_DEV void load4_16(const H* __restrict__ x, int i, int hi, bool vec, float* o) {
    if (vec && i + 3 < hi) {
        const uint2 v = __ldg(reinterpret_cast<const uint2*>(x + i));
        const H* h = reinterpret_cast<const H*>(&v);
#pragma unroll
        for (int j = 0; j < 4; ++j) o[j] = to_f32<H>(h[j]);
        return;
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) o[j] = i + j < hi ? to_f32<H>(x[i + j]) : -INFINITY;
}
template <>
SDL_DEV void load4<__nv_bfloat16>(const __nv_bfloat16* __restrict__ x, int i, int hi, bool vec, float* o) {
    load4_16<__nv_bfloat16>(x, i, hi, vec, o);
}
template <>
SDL_DEV void load4<__half>(const __half* __restrict__ x, int i, int hi, bool vec, float* o) {
    load4_16<__half>(x, i, hi, vec, o);
}

template <typename T>
SDL_DEV bool row_vec_ok(const T* x) { return reinterpret_cast<uintptr_t>(x) % (4 * sizeof(T)) == 0; }

// p_i from the scaled logit and the row statistics (m, r = 1/s).
SDL_DEV float prob_of(float xs, float m, float r) { return __fmul_rn(expf(__fsub_rn(xs, m)), r); }

// Statistics (m_c, s_c) of elements [lo, hi) of row x, reduced by one
// 256-thread group (g = thread index in the group, bar_id its named barrier,
// red = 8 floats of group-private shared memory).  Valid in every thread.
template <typename T>
SDL_DEV float2 chunk_stats(const T* __restrict__ x, int lo, int hi, float temp, int g, int bar_id, float* red) {
    float v[kPerThread];
    float mt = -INFINITY;
    const bool vec = row_vec_ok<T>(x);
#pragma unroll
    for (int k = 0; k < kPerThread / 4; ++k) load4<T>(x, lo + 4 * g + 1024 * k, hi, vec, v + 4 * k);
    if (temp != 1.f) {
#pragma unroll
        for (int e = 0; e < kPerThread; ++e) v[e] = __fdiv_rn(v[e], temp);
    }
#pragma unroll
    for (int e = 0; e < kPerThread; ++e) mt = fmaxf(mt, v[e]);
    const int lane = g & 31, w = g >> 5;
    mt = warp_max(mt);
    if (lane == 0) red[w] = mt;
    group_sync(bar_id);
    float mc = red[0];
#pragma unroll
    for (int i = 1; i < kGroup / 32; ++i) mc = fmaxf(mc, red[i]);
    group_sync(bar_id);
    float st = 0.f;
    if (mc != -INFINITY) {
#pragma unroll
        for (int e = 0; e < kPerThread; ++e) st = __fadd_rn(st, expf(__fsub_rn(v[e], mc)));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) st = __fadd_rn(st, __shfl_xor_sync(0xffffffffu, st, o));
    if (lane == 0) red[w] = st;
    group_sync(bar_id);
    float sc = red[0];
#pragma unroll
    for (int i = 1; i < kGroup / 32; ++i) sc = __fadd_rn(sc, red[i]);
    group_sync(bar_id);
    return make_float2(mc, sc);
}

// Sequential merge of a row's chunk statistics (one thread).
SDL_DEV float2 merge_stats(const float2* st, int nchunks) {
    float m = -INFINITY;
    for (int c = 0; c < nchunks; ++c) m = fmaxf(m, st[c].x);
    float s = 0.f;
    if (m != -INFINITY)
        for (int c = 0; c < nchunks; ++c)
            if (st[c].x != -INFINITY) s = __fmaf_rn(st[c].y, expf(__fsub_rn(st[c].x, m)), s);
    return make_float2(m, s);
}

// ------------------------------------------------------------ probabilities
// One CTA (4 groups of 256) per row: chunk statistics, merge, then p_i.
template <typename T>
__global__ void __launch_bounds__(1024) probs_canon_kernel(const T* __restrict__ logits, int64_t row_stride, int V,
                                                           float temp, float* __restrict__ out, int64_t out_stride) {
    __shared__ float red[4][8];
    __shared__ float2 s_st[kMaxChunks];
    __shared__ float2 s_row;
    const T* x = logits + blockIdx.x * row_stride;
    float* o = out + blockIdx.x * out_stride;
    const int grp = threadIdx.x / kGroup, g = threadIdx.x % kGroup;
    const int nchunks = (V + kChunk - 1) / kChunk;
    for (int c = grp; c < nchunks; c += 4) {
        const float2 st = chunk_stats<T>(x, c * kChunk, min(V, (c + 1) * kChunk), temp, g, 1 + grp, red[grp]);
        if (g == 0) s_st[c] = st;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        const float2 ms = merge_stats(s_st, nchunks);
        s_row = make_float2(ms.x, __frcp_rn(ms.y));
    }
    __syncthreads();
    const float m = s_row.x, r = s_row.y;
    for (int i = threadIdx.x; i < V; i += blockDim.x) o[i] = prob_of(scaled(to_f32<T>(x[i]), temp), m, r);
}

// Chunk statistics of every (row, chunk); rows [0, A.n) come from A and
// [A.n, A.n + Bq.n) from Bq.  Grid (nchunks, A.n + Bq.n), 256 threads.
template <typename T>
__global__ void __launch_bounds__(kGroup) stats_kernel(Rows<T> A, Rows<T> Bq, int V, float temp, float2* stats) {
    __shared__ float red[8];
    pdl_wait();
    pdl_launch_dependents();
    const int r = blockIdx.y, c = blockIdx.x;
    const T* x = r < A.n ? A.row(r) : Bq.row(r - A.n);
    const float2 st = chunk_stats<T>(x, c * kChunk, min(V, (c + 1) * kChunk), temp, threadIdx.x, 1, red);
    if (threadIdx.x == 0) stats[(int64_t)r * gridDim.x + c] = st;
}

// Row statistics (m, 1/s) from the chunk statistics of every row: the chunk
// entries are loaded in parallel, the maximum is reduced in any order (it is
// exact), the rescale factors are evaluated in parallel and thread 0 adds
// them in chunk order -- the operations of merge_stats.  Grid rows, 128
// threads.
__global__ void __launch_bounds__(128) merge_kernel(const float2* __restrict__ stats, int nchunks,
                                                    float2* __restrict__ rowstat) {
    __shared__ float2 s_st[kMaxChunks];
    __shared__ float s_fac[kMaxChunks];
    __shared__ float s_red[4];
    pdl_wait();
    pdl_launch_dependents();
    const int r = blockIdx.x;
    const float2* st = stats + (int64_t)r * nchunks;
    float m = -INFINITY;
    for (int c = threadIdx.x; c < nchunks; c += blockDim.x) {
        const float2 v = st[c];
        s_st[c] = v;
        m = fmaxf(m, v.x);
    }
    m = warp_max(m);
    if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = m;
    __syncthreads();
    m = fmaxf(fmaxf(s_red[0], s_red[1]), fmaxf(s_red[2], s_red[3]));
    for (int c = threadIdx.x; c < nchunks; c += blockDim.x)
        s_fac[c] = s_st[c].x != -INFINITY ? expf(__fsub_rn(s_st[c].x, m)) : 0.f;
    __syncthreads();
    if (threadIdx.x == 0) {
        float s = 0.f;
        if (m != -INFINITY)
            for (int c = 0; c < nchunks; ++c)
                if (s_st[c].x != -INFINITY) s = __fmaf_rn(s_st[c].y, s_fac[c], s);
        rowstat[r] = make_float2(m, __frcp_rn(s));
    }
}

// Inclusive block scan of one u64 per thread (blockDim a multiple of 32).
SDL_DEV uint64_t block_incl_scan_u64(uint64_t v, uint64_t* s_w /*[32]*/, uint64_t* total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    uint64_t x = warp_incl_scan_u64(v, lane);
    if (lane == 31) s_w[warp] = x;
    __syncthreads();
    uint64_t off = 0, tot = 0;
    for (int w = 0; w < nw; ++w) {
        if (w < warp) off += s_w[w];
        tot += s_w[w];
    }
    __syncthreads();
    *total = tot;
    return off + x;
}

// ----------------------------------------------------------------- draws
// What one draw row samples from.
//   kind 0: p of logits row pr (plain draw)
//   kind 1: residual clamp(p - q, 0) of rows pr / qr, with p as fallback
struct DrawRow {
    int kind;
    int pr, qr;  // statistics row indices
};

// Per-slice exact integer weight sums of each draw's distribution (p, or the
// residual clamp(p - q, 0) for a rejected proposal).  Grid (nchunks = draw
// slices, n_draw), 256 threads: wsum[d][c] = sum of W over slice c.
template <typename T>
__global__ void __launch_bounds__(kGroup) wsum_kernel(Rows<T> A, Rows<T> Bq, int V, float temp,
                                                      const float2* __restrict__ rowstat, int nchunks, int mode,
                                                      int gamma, const int* __restrict__ n_acc, uint64_t* wsum) {
    __shared__ uint64_t red[8];
    pdl_wait();
    pdl_launch_dependents();
    const int d = blockIdx.y, c = blockIdx.x;
    // mode 0: draw d samples p of row d (A).  mode 1: spec round of sequence d.
    int pr, qr = -1;
    if (mode == 0) {
        pr = d;
    } else {
        const int r = n_acc[d];
        pr = d * (gamma + 1) + r;                         // target row r of sequence d
        if (r < gamma) qr = A.n + d * gamma + r;          // draft row r (stats rows after A's)
    }
    const float2 sp = rowstat[pr];
    const float2 sq = qr >= 0 ? rowstat[qr] : make_float2(0.f, 1.f);
    const T* xp = A.row(pr);
    const T* xq = qr >= 0 ? Bq.row(qr - A.n) : nullptr;
    const int lo = c * kDrawChunk, hi = min(V, lo + kDrawChunk);
    // every load of the thread's slice in flight before any arithmetic
    float vp[kDrawPerThread], vq[kDrawPerThread];
    const bool vecp = row_vec_ok<T>(xp);
#pragma unroll
    for (int k = 0; k < kDrawPerThread / 4; ++k) load4<T>(xp, lo + 4 * threadIdx.x + 1024 * k, hi, vecp, vp + 4 * k);
    if (xq) {
        const bool vecq = row_vec_ok<T>(xq);
#pragma unroll
        for (int k = 0; k < kDrawPerThread / 4; ++k)
            load4<T>(xq, lo + 4 * threadIdx.x + 1024 * k, hi, vecq, vq + 4 * k);
    }
    uint64_t w = 0;
    if (xq) {
#pragma unroll
        for (int e = 0; e < kDrawPerThread; ++e) {
            const float p = prob_of(scaled(vp[e], temp), sp.x, sp.y);
            const float q = prob_of(scaled(vq[e], temp), sq.x, sq.y);
            w += wfix(fmaxf(__fsub_rn(p, q), 0.f));
        }
    } else {
#pragma unroll
        for (int e = 0; e < kDrawPerThread; ++e) w += wfix(prob_of(scaled(vp[e], temp), sp.x, sp.y));
    }
    w = warp_sum_u64(w);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = w;
    __syncthreads();
    if (threadIdx.x == 0) {
        uint64_t a = 0;
        for (int i = 0; i < kGroup / 32; ++i) a += red[i];
        wsum[(int64_t)d * nchunks + c] = a;
    }
}

// First index i in [lo, hi) whose prefix (from lo) of W exceeds `target`.
// Whole CTA (1024 threads); warps own contiguous ranges.
template <typename WF>
SDL_DEV int block_find(WF wf, int lo, int hi, uint64_t target, uint64_t* s_w, int* s_tok) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    int seg = (hi - lo + nw - 1) / nw;
    seg = (seg + 31) & ~31;
    const int a = lo + warp * seg, b = min(hi, a + seg);
    uint64_t s = 0;
    for (int i = a + lane; i < b; i += 32) s += wfix(wf(i));
    s = warp_sum_u64(s);
    if (lane == 0) s_w[warp] = s;
    if (threadIdx.x == 0) *s_tok = -1;
    __syncthreads();
    uint64_t excl = 0;
    for (int w = 0; w < warp; ++w) excl += s_w[w];
    if (excl <= target && target < excl + s_w[warp]) {
        uint64_t run = excl;
        for (int base = a; base < b; base += 32) {
            const int i = base + lane;
            const uint64_t val = i < b ? wfix(wf(i)) : 0ull;
            const uint64_t pre = warp_incl_scan_u64(val, lane);
            const unsigned hit = __ballot_sync(0xffffffffu, run + pre > target);
            if (hit) {
                if (lane == 0) *s_tok = base + __ffs(hit) - 1;
                break;
            }
            run += __shfl_sync(0xffffffffu, pre, 31);
        }
    }
    __syncthreads();
    const int t = *s_tok;
    __syncthreads();
    return t;
}

// Finish every draw: total of the chunk sums, the residual fallback test,
// the target, the chunk holding it, then the index inside that chunk.
// Grid n_draw, 1024 threads.
template <typename T>
__global__ void __launch_bounds__(1024) finish_kernel(Rows<T> A, Rows<T> Bq, int V, float temp,
                                                      const float2* __restrict__ rowstat, int nchunks, int mode,
                                                      int gamma, const int* __restrict__ n_acc,
                                                      const int* __restrict__ u_bits, const float* __restrict__ uniforms,
                                                      int64_t nu, const int64_t* u_base, int64_t u_off,
                                                      const uint64_t* __restrict__ wsum, uint64_t* wsum_p,
                                                      const int* __restrict__ prop, int* out, int* n_out, int* err) {
    __shared__ uint64_t s_w[32];
    __shared__ int s_tok, s_chunk;
    __shared__ uint64_t s_target;
    pdl_wait();
    const int d = blockIdx.x;
    int pr, qr = -1, r = 0;
    float u;
    if (mode == 0) {
        pr = d;
        const int64_t ui = (u_base ? *u_base : 0) + u_off + d;
        if (ui < 0 || ui >= nu) {
            if (threadIdx.x == 0) { sdl_raise(err, SDL_DEVERR_UNIFORMS); out[d] = 0; }
            return;
        }
        u = uniforms[ui];
    } else {
        r = n_acc[d];
        pr = d * (gamma + 1) + r;
        if (r < gamma) qr = A.n + d * gamma + r;
        u = __int_as_float(u_bits[d]);
    }
    const uint64_t* ws = wsum + (int64_t)d * nchunks;
    // slice sums (one slice per thread; nchunks <= blockDim) and their total
    const int c = threadIdx.x;
    uint64_t wc = c < nchunks ? ws[c] : 0ull;
    uint64_t S;
    uint64_t incl = block_incl_scan_u64(wc, s_w, &S);
    bool usep = false;
    if (qr >= 0 && (double)S / kTwo62 <= 1e-12) {
        // residual mass <= 1e-12 (rare): draw from p; its slice sums are made
        // here, one warp per slice
        usep = true;
        const float2 sp = rowstat[pr];
        const T* xp = A.row(pr);
        const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
        for (int sl = warp; sl < nchunks; sl += blockDim.x >> 5) {
            const int lo = sl * kDrawChunk, hi = min(V, lo + kDrawChunk);
            uint64_t a = 0;
            for (int i = lo + lane; i < hi; i += 32) a += wfix(prob_of(scaled(to_f32<T>(xp[i]), temp), sp.x, sp.y));
            a = warp_sum_u64(a);
            if (lane == 0) wsum_p[(int64_t)d * nchunks + sl] = a;
        }
        __threadfence_block();
        __syncthreads();
        wc = c < nchunks ? wsum_p[(int64_t)d * nchunks + c] : 0ull;
        incl = block_incl_scan_u64(wc, s_w, &S);
    }
    if (threadIdx.x == 0) s_chunk = -1;
    __syncthreads();
    const uint64_t target = S != 0 ? __umul64hi(ufix(u), S) : 0ull;
    if (S != 0 && wc != 0 && incl - wc <= target && target < incl) {  // the chunk holding the target
        s_chunk = c;
        s_target = target - (incl - wc);
    }
    __syncthreads();
    const int chunk = s_chunk;
    int tok = -1;
    if (chunk >= 0) {
        const float2 sp = rowstat[pr];
        const T* xp = A.row(pr);
        const int lo = chunk * kDrawChunk, hi = min(V, lo + kDrawChunk);
        if (qr >= 0 && !usep) {
            const float2 sq = rowstat[qr];
            const T* xq = Bq.row(qr - A.n);
            tok = block_find(
                [&](int i) {
                    const float p = prob_of(scaled(to_f32<T>(xp[i]), temp), sp.x, sp.y);
                    const float q = prob_of(scaled(to_f32<T>(xq[i]), temp), sq.x, sq.y);
                    return fmaxf(__fsub_rn(p, q), 0.f);
                },
                lo, hi, s_target, s_w, &s_tok);
        } else {
            tok = block_find([&](int i) { return prob_of(scaled(to_f32<T>(xp[i]), temp), sp.x, sp.y); }, lo, hi,
                             s_target, s_w, &s_tok);
        }
    }
    if (threadIdx.x == 0) {
        if (tok < 0) { sdl_raise(err, SDL_DEVERR_BAD_SAMPLE); tok = 0; }
        if (mode == 0) {
            out[d] = tok;
        } else {
            for (int j = 0; j < r; ++j) out[d * (gamma + 1) + j] = prop[d * gamma + j];
            out[d * (gamma + 1) + r] = tok;
            n_out[d] = r + 1;
        }
    }
}

// Accept walk of a speculative round from logits (one CTA): acceptance
// probabilities min(1, p/q) in fp64 from the canonical p_x, q_x
// (specdec/sampler.py:86-92), then the reference's uniform consumption
// (engine/spec_scheduler.py:67-87): per sequence one uniform per accept
// test, plus one for the residual or bonus draw.
template <typename T>
__global__ void __launch_bounds__(1024) accept_logits_kernel(Rows<T> A, Rows<T> Bq, int V, float temp,
                                                             const float2* __restrict__ rowstat,
                                                             const int* __restrict__ prop, int B, int gamma,
                                                             const float* __restrict__ uniforms, int64_t nu,
                                                             int64_t* u_base, int64_t u_skip, int* n_acc,
                                                             int* u_bits, int* err, const int* n_valid) {
    extern __shared__ double s_dyn[];
    double* a = s_dyn;                                                // [B*gamma]
    float* uc = reinterpret_cast<float*>(s_dyn + (size_t)B * gamma);  // [B*(gamma+1)]
    pdl_wait();
    const int64_t base = (u_base ? *u_base : 0) + u_skip;
    // sequences past *n_valid pad a captured batch: no uniforms, a harmless bonus draw
    const int Bn = n_valid != nullptr ? min(B, max(0, *n_valid)) : B;
    for (int idx = threadIdx.x; idx < B * gamma; idx += blockDim.x) {
        const int b = idx / gamma, j = idx % gamma;
        const int x = prop[idx];
        if (x < 0 || x >= V) {  // a proposal outside the vocabulary is rejected
            sdl_raise(err, SDL_DEVERR_BAD_INDEX);
            a[idx] = 0.0;
            continue;
        }
        const int pr = b * (gamma + 1) + j, qr = A.n + idx;
        const float2 sp = rowstat[pr];
        const float2 sq = rowstat[qr];
        const double pv = prob_of(scaled(to_f32<T>(A.row(pr)[x]), temp), sp.x, sp.y);
        const double qv = prob_of(scaled(to_f32<T>(Bq.row(idx)[x]), temp), sq.x, sq.y);
        double acc;
        if (qv <= 1e-12) acc = pv > 1e-12 ? 1.0 : 0.0;
        else acc = fmin(1.0, pv / qv);
        a[idx] = acc;
    }
    for (int i = threadIdx.x; i < B * (gamma + 1); i += blockDim.x) {
        const int64_t ui = base + i;
        uc[i] = (ui >= 0 && ui < nu) ? uniforms[ui] : __int_as_float(0x7fc00000);
    }
    __syncthreads();
    if (threadIdx.x >= 32) return;
    const int lane = threadIdx.x;
    int off = 0;
    bool bad_u = false;
    for (int b = Bn + lane; b < B; b += 32) {
        n_acc[b] = gamma;
        u_bits[b] = __float_as_int(0.5f);
    }
    for (int b = 0; b < Bn; ++b) {
        bool reject = false;
        if (lane < gamma) {
            const float u = uc[off + lane];
            if (u != u) bad_u = true;
            reject = !((double)u < a[b * gamma + lane]);
        }
        const unsigned rj = __ballot_sync(0xffffffffu, reject);
        const int r = rj ? __ffs(rj) - 1 : gamma;
        const int consumed = r < gamma ? r + 2 : gamma + 1;
        if (lane == 0) {
            n_acc[b] = r;
            const float uf = uc[off + consumed - 1];
            if (uf != uf) bad_u = true;
            u_bits[b] = __float_as_int(uf);
        }
        off += consumed;
    }
    bad_u = __any_sync(0xffffffffu, bad_u);
    if (lane == 0) {
        if (bad_u) sdl_raise(err, SDL_DEVERR_UNIFORMS);
        if (u_base) *u_base = base + off;
    }
}

// -------------------------------------------- fused rejection sampling
// spec_fused_kernel: the whole speculative sampling step of a round in one
// launch -- softmax statistics of every p and q row, the fp64 accept tests
// with the reference's uniform consumption, and the residual / bonus draw --
// with the same operations as the stats -> merge -> accept -> wsum -> finish
// chain above, so tokens, accept lengths and the stream counter are
// bit-identical to it.
//
// One thread-block cluster of up to kFuseCluster CTAs (two 256-thread
// groups each, working on separate chunks) per sequence b:
//  1. the cluster's CTAs take the (row, 8192-chunk) statistics of the
//     sequence's 2*gamma+1 logit rows (chunk_stats) into the workspace;
//  2. after a cluster barrier, CTA 0 merges each row (merge_kernel's order),
//     computes min(1, p/q) for its gamma proposals (accept_logits_kernel's
//     arithmetic), publishes them and a flag, then waits -- bounded -- for
//     the flags of sequences 0..b-1 and walks their accept tests in order
//     to find where this sequence's uniforms start in the stream (the
//     reference draws them sequence after sequence); the last sequence also
//     advances the stream counter;
//  3. the cluster's CTAs sum the integer weights W of the drawn
//     distribution -- (p_r - q_r)+ after a rejection at r, else p_gamma --
//     per 2048-element slice; CTA 0 finds the slice and the token
//     (finish_kernel's rule).
// The only wait on another cluster is step 2's, and only on lower sequence
// numbers; the host launches this kernel only when every cluster of the
// grid can be resident at once, so that wait always ends (it is bounded
// all the same).  Flags carry a launch epoch kept in the workspace's
// control block with a done counter; the last cluster to finish advances
// the epoch, so the flags never need clearing.
constexpr int kFuseCluster = 8;
constexpr size_t kCtrlBytes = 64 * 1024;              // control block at the start of the sampler workspace
constexpr int kCtrlWords = 16;                        // [0] epoch, [1] done counter
constexpr int kMaxFusedSeqs = (int)(kCtrlBytes / 4) - kCtrlWords;
constexpr uint32_t kFlagWaitLimit = 1u << 22;          // polls, 64 ns apart
constexpr int kMaxFusedRows = 65;                       // 2 * gamma + 1 for gamma <= 32
constexpr int kFuseGroups = 2;                          // 256-thread groups per CTA (chunk tasks in flight)
constexpr int kFuseThreads = kFuseGroups * kGroup;
constexpr int kFuseMaxDrawChunks = kFuseThreads;        // draw slices CTA 0 scans with one value per thread

struct FusedWs {
    float2* stats;    // [B][R][nchunks]
    float2* rowstat;  // [B][R] (m, 1/s)
    double* acc;      // [B][gamma]
    uint64_t* wsum;   // [B][ndc]
    uint64_t* wsum_p; // [B][ndc] (residual fallback)
    int* ctrl;        // [0] epoch, [1] done, then flags[B] from kCtrlWords
};

SDL_DEV int ld_acquire_i32(const int* p) {
    int v;
    asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

SDL_DEV void st_release_i32(int* p, int v) {
    asm volatile("st.release.gpu.global.b32 [%0], %1;" :: "l"(p), "r"(v) : "memory");
}

SDL_DEV int ld_cluster_i32(uint32_t addr) {
    int v;
    asm volatile("ld.shared::cluster.b32 %0, [%1];" : "=r"(v) : "r"(addr) : "memory");
    return v;
}

template <typename T>
__global__ void __launch_bounds__(kFuseThreads, 2) spec_fused_kernel(Rows<T> A, Rows<T> Q, int V, float temp,
                                                            const int* __restrict__ prop, int B, int gamma,
                                                            const float* __restrict__ uniforms, int64_t nu,
                                                            int64_t* u_base, int64_t u_skip, int* tokens, int* n_out,
                                                            FusedWs w, int nchunks, int ndc, int* err) {
    extern __shared__ double s_walk[];  // CTA 0: acceptance of sequences 0..b, then their uniforms
    __shared__ float red[kFuseGroups][8];
    __shared__ uint64_t s_wg[kFuseGroups][8];
    __shared__ float2 s_rs[kMaxFusedRows];
    __shared__ uint64_t s_w[32];
    __shared__ int s_tok, s_chunk, s_r, s_ok, s_epoch;
    __shared__ float s_u;
    __shared__ uint64_t s_target;
    __shared__ int64_t s_base;
    pdl_wait();
    const int cs = gridDim.x;  // CTAs per sequence (the cluster)
    const int rank = (int)cluster_ctarank();
    const int b = blockIdx.y;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int grp = tid / kGroup, g = tid % kGroup;  // the CTA's 256-thread groups work on separate chunks
    const int R = 2 * gamma + 1;
    int* flags = w.ctrl + kCtrlWords;
    if (rank == 0 && tid == 0) {
        // read before any cluster of this launch can change them: the epoch
        // moves and the counter is written only after every cluster is done
        s_epoch = ld_acquire_i32(w.ctrl);
        s_base = (u_base ? *u_base : 0) + u_skip;
    }

    // 1. chunk statistics of the sequence's rows: p rows 0..gamma, then q rows
    for (int t = rank * kFuseGroups + grp; t < R * nchunks; t += cs * kFuseGroups) {
        const int row = t / nchunks, c = t % nchunks;
        const T* x = row <= gamma ? A.row(b * (gamma + 1) + row) : Q.row(b * gamma + row - gamma - 1);
        const float2 st = chunk_stats<T>(x, c * kChunk, min(V, (c + 1) * kChunk), temp, g, 1 + grp, red[grp]);
        if (g == 0) w.stats[((int64_t)b * R + row) * nchunks + c] = st;
    }
    __threadfence();
    cluster_sync_all();

    if (rank == 0) {
        // 2a. row statistics (m, 1/s): merge_kernel's operations, one warp per row
        for (int row = warp; row < R; row += kFuseThreads / 32) {
            const float2* st = w.stats + ((int64_t)b * R + row) * nchunks;
            float m = -INFINITY;
            for (int c = lane; c < nchunks; c += 32) m = fmaxf(m, __ldcg(st + c).x);
            m = warp_max(m);
            float s = 0.f;
            if (m != -INFINITY) {
                for (int c0 = 0; c0 < nchunks; c0 += 32) {
                    const float2 v = c0 + lane < nchunks ? __ldcg(st + c0 + lane) : make_float2(-INFINITY, 0.f);
                    const float f = v.x != -INFINITY ? expf(__fsub_rn(v.x, m)) : 0.f;
                    const int n = min(32, nchunks - c0);
                    for (int k = 0; k < n; ++k) {  // chunk order, as merge_kernel's thread 0
                        const float vx = __shfl_sync(0xffffffffu, v.x, k);
                        const float vy = __shfl_sync(0xffffffffu, v.y, k);
                        const float fk = __shfl_sync(0xffffffffu, f, k);
                        if (vx != -INFINITY) s = __fmaf_rn(vy, fk, s);
                    }
                }
            }
            if (lane == 0) {
                const float2 rs = make_float2(m, __frcp_rn(s));
                s_rs[row] = rs;
                w.rowstat[(int64_t)b * R + row] = rs;
            }
        }
        __syncthreads();
        // 2b. min(1, p/q) of this sequence's proposals (accept_logits_kernel's arithmetic)
        if (tid < gamma) {
            const int x = prop[b * gamma + tid];
            double acc;
            if (x < 0 || x >= V) {  // a proposal outside the vocabulary is rejected
                sdl_raise(err, SDL_DEVERR_BAD_INDEX);
                acc = 0.0;
            } else {
                const float2 sp = s_rs[tid], sq = s_rs[gamma + 1 + tid];
                const double pv = prob_of(scaled(to_f32<T>(A.row(b * (gamma + 1) + tid)[x]), temp), sp.x, sp.y);
                const double qv = prob_of(scaled(to_f32<T>(Q.row(b * gamma + tid)[x]), temp), sq.x, sq.y);
                if (qv <= 1e-12) acc = pv > 1e-12 ? 1.0 : 0.0;
                else acc = fmin(1.0, pv / qv);
            }
            w.acc[(int64_t)b * gamma + tid] = acc;
        }
        __syncthreads();
        if (tid == 0) {
            __threadfence();
            st_release_i32(flags + b, s_epoch + 1);
        }
        // 2c. where this sequence's uniforms start: the tests of sequences
        // 0..b-1 (bounded wait for their flags), walked in order
        int ok = 1;
        for (int bp = tid; bp < b && ok; bp += kFuseThreads) {
            uint32_t n = 0;
            while (ld_acquire_i32(flags + bp) != s_epoch + 1) {
                if (++n > kFlagWaitLimit) { ok = 0; break; }
                __nanosleep(64);
            }
        }
        ok = __syncthreads_and(ok);
        double* a_s = s_walk;                                                      // [(b+1) * gamma]
        float* u_s = reinterpret_cast<float*>(s_walk + (size_t)(b + 1) * gamma);  // [(b+1) * (gamma+1)]
        const int64_t base = s_base;
        if (ok) {
            for (int i = tid; i < (b + 1) * gamma; i += kFuseThreads) a_s[i] = __ldcg(w.acc + i);
            for (int i = tid; i < (b + 1) * (gamma + 1); i += kFuseThreads) {
                const int64_t ui = base + i;
                u_s[i] = (ui >= 0 && ui < nu) ? uniforms[ui] : __int_as_float(0x7fc00000);
            }
        }
        __syncthreads();
        if (warp == 0) {
            int off = 0, r = 0;
            float uf = 0.5f;
            bool bad_u = false;
            if (ok) {
                for (int bb = 0; bb <= b; ++bb) {
                    bool reject = false;
                    if (lane < gamma) {
                        const float u = u_s[off + lane];
                        if (u != u) bad_u = true;
                        reject = !((double)u < a_s[bb * gamma + lane]);
                    }
                    const unsigned rj = __ballot_sync(0xffffffffu, reject);
                    r = rj ? __ffs(rj) - 1 : gamma;
                    const int consumed = r < gamma ? r + 2 : gamma + 1;
                    uf = u_s[off + consumed - 1];
                    if (uf != uf) bad_u = true;
                    off += consumed;
                }
            }
            bad_u = __any_sync(0xffffffffu, bad_u);
            if (lane == 0) {
                if (!ok) sdl_raise(err, SDL_DEVERR_TIMEOUT);
                if (bad_u) sdl_raise(err, SDL_DEVERR_UNIFORMS);
                s_r = ok ? r : 0;
                s_u = uf;
                s_ok = ok;
                if (ok && b == B - 1 && u_base) *u_base = base + off;
            }
        }
    }
    cluster_sync_all();  // r and u (and the row statistics) for the whole cluster
    int r;
    float u;
    if (rank == 0) {
        r = s_r;
        u = s_u;
    } else {
        r = ld_cluster_i32(mapa_shared(smem_u32(&s_r), 0));
        u = ld_cluster_f32(mapa_shared(smem_u32(&s_u), 0));
    }

    // 3. the draw: integer weight sums of its distribution per 2048-element
    // slice (wsum_kernel's operations), over the cluster's CTAs
    const int prow = r;                                 // p row r of the sequence
    const int qrow = r < gamma ? gamma + 1 + r : -1;    // q row r, or none after a full accept
    const float2 sp = __ldcg(w.rowstat + (int64_t)b * R + prow);
    const float2 sq = qrow >= 0 ? __ldcg(w.rowstat + (int64_t)b * R + qrow) : make_float2(0.f, 1.f);
    const T* xp = A.row(b * (gamma + 1) + r);
    const T* xq = qrow >= 0 ? Q.row(b * gamma + r) : nullptr;
    for (int c = rank * kFuseGroups + grp; c < ndc; c += cs * kFuseGroups) {
        const int lo = c * kDrawChunk, hi = min(V, lo + kDrawChunk);
        float vp[kDrawPerThread], vq[kDrawPerThread];
        const bool vecp = row_vec_ok<T>(xp);
#pragma unroll
        for (int k = 0; k < kDrawPerThread / 4; ++k) load4<T>(xp, lo + 4 * g + 1024 * k, hi, vecp, vp + 4 * k);
        if (xq) {
            const bool vecq = row_vec_ok<T>(xq);
#pragma unroll
            for (int k = 0; k < kDrawPerThread / 4; ++k) load4<T>(xq, lo + 4 * g + 1024 * k, hi, vecq, vq + 4 * k);
        }
        uint64_t wt = 0;
        if (xq) {
#pragma unroll
            for (int e = 0; e < kDrawPerThread; ++e) {
                const float p = prob_of(scaled(vp[e], temp), sp.x, sp.y);
                const float q = prob_of(scaled(vq[e], temp), sq.x, sq.y);
                wt += wfix(fmaxf(__fsub_rn(p, q), 0.f));
            }
        } else {
#pragma unroll
            for (int e = 0; e < kDrawPerThread; ++e) wt += wfix(prob_of(scaled(vp[e], temp), sp.x, sp.y));
        }
        wt = warp_sum_u64(wt);
        if (lane == 0) s_wg[grp][g >> 5] = wt;
        group_sync(1 + grp);
        if (g == 0) {
            uint64_t a = 0;
            for (int i = 0; i < kGroup / 32; ++i) a += s_wg[grp][i];
            w.wsum[(int64_t)b * ndc + c] = a;
        }
        group_sync(1 + grp);
    }
    __threadfence();
    cluster_sync_all();
    if (rank != 0) return;

    // CTA 0: the slice holding the target and the token in it (finish_kernel's rule)
    const uint64_t* ws = w.wsum + (int64_t)b * ndc;
    const int c = tid;
    uint64_t wc = c < ndc ? __ldcg(ws + c) : 0ull;
    uint64_t S;
    uint64_t incl = block_incl_scan_u64(wc, s_w, &S);
    bool usep = false;
    if (qrow >= 0 && (double)S / kTwo62 <= 1e-12) {
        // residual mass <= 1e-12 (rare): draw from p; its slice sums, one warp per slice
        usep = true;
        for (int sl = warp; sl < ndc; sl += kFuseThreads / 32) {
            const int lo = sl * kDrawChunk, hi = min(V, lo + kDrawChunk);
            uint64_t a = 0;
            for (int i = lo + lane; i < hi; i += 32) a += wfix(prob_of(scaled(to_f32<T>(xp[i]), temp), sp.x, sp.y));
            a = warp_sum_u64(a);
            if (lane == 0) w.wsum_p[(int64_t)b * ndc + sl] = a;
        }
        __threadfence_block();
        __syncthreads();
        wc = c < ndc ? w.wsum_p[(int64_t)b * ndc + c] : 0ull;
        incl = block_incl_scan_u64(wc, s_w, &S);
    }
    if (tid == 0) s_chunk = -1;
    __syncthreads();
    const uint64_t target = S != 0 ? __umul64hi(ufix(u), S) : 0ull;
    if (S != 0 && wc != 0 && incl - wc <= target && target < incl) {
        s_chunk = c;
        s_target = target - (incl - wc);
    }
    __syncthreads();
    const int chunk = s_chunk;
    int tok = -1;
    if (chunk >= 0) {
        const int lo = chunk * kDrawChunk, hi = min(V, lo + kDrawChunk);
        if (xq && !usep) {
            tok = block_find(
                [&](int i) {
                    const float p = prob_of(scaled(to_f32<T>(xp[i]), temp), sp.x, sp.y);
                    const float q = prob_of(scaled(to_f32<T>(xq[i]), temp), sq.x, sq.y);
                    return fmaxf(__fsub_rn(p, q), 0.f);
                },
                lo, hi, s_target, s_w, &s_tok);
        } else {
            tok = block_find([&](int i) { return prob_of(scaled(to_f32<T>(xp[i]), temp), sp.x, sp.y); }, lo, hi,
                             s_target, s_w, &s_tok);
        }
    }
    if (tid == 0) {
        if (tok < 0) { sdl_raise(err, SDL_DEVERR_BAD_SAMPLE); tok = 0; }
        for (int j = 0; j < r; ++j) tokens[b * (gamma + 1) + j] = prop[b * gamma + j];
        tokens[b * (gamma + 1) + r] = tok;
        n_out[b] = r + 1;
        // launch bookkeeping: the last cluster to get here moves the epoch on
        __threadfence();
        if (atomicAdd(w.ctrl + 1, 1) == B - 1) {
            w.ctrl[1] = 0;
            __threadfence();
            st_release_i32(w.ctrl, s_epoch + 1);
        }
    }
}

// ------------------------------------------------------------ host side
struct Ws {
    float2* stats;
    float2* rowstat;
    uint64_t* wsum;
    uint64_t* wsum_p;
    int* n_acc;
    int* u_bits;
    size_t bytes;
};

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// Every sampler workspace starts with the fused kernel's control block
// (launch epoch, done counter, per-sequence flags), which must be zero before
// a workspace's first use; no kernel of the chain touches it.
Ws carve(void* base, int stat_rows, int draws, int nchunks, int ndc) {
    Ws w;
    char* p = static_cast<char*>(base);
    size_t o = kCtrlBytes;
    w.stats = reinterpret_cast<float2*>(p + o);
    o = align256(o + (size_t)stat_rows * nchunks * sizeof(float2));
    w.rowstat = reinterpret_cast<float2*>(p + o);
    o = align256(o + (size_t)stat_rows * sizeof(float2));
    w.wsum = reinterpret_cast<uint64_t*>(p + o);
    o = align256(o + (size_t)draws * ndc * sizeof(uint64_t));
    w.wsum_p = reinterpret_cast<uint64_t*>(p + o);
    o = align256(o + (size_t)draws * ndc * sizeof(uint64_t));
    w.n_acc = reinterpret_cast<int*>(p + o);
    o = align256(o + (size_t)draws * sizeof(int));
    w.u_bits = reinterpret_cast<int*>(p + o);
    o = align256(o + (size_t)draws * sizeof(int));
    w.bytes = o;
    return w;
}

template <typename T>
int sample_logits_t(const T* logits, int64_t row_stride, int rows, int V, float temp, const float* uniforms, int64_t nu,
                    const int64_t* u_base, int64_t u_off, int* out, void* ws_base, int* err, cudaStream_t st) {
    const int nchunks = (V + kChunk - 1) / kChunk;
    const int ndc = (V + kDrawChunk - 1) / kDrawChunk;
    Ws w = carve(ws_base, rows, rows, nchunks, ndc);
    Rows<T> A{logits, row_stride, 0, 1, rows};
    Rows<T> none{logits, 0, 0, 1, 0};
    cudaError_t e = sdl::launch_pdl(stats_kernel<T>, dim3(nchunks, rows), dim3(kGroup), 0, st, A, none, V, temp,
                                    w.stats);
    if (e == cudaSuccess)
        e = sdl::launch_pdl(merge_kernel, dim3(rows), dim3(128), 0, st, (const float2*)w.stats, nchunks, w.rowstat);
    if (e == cudaSuccess)
        e = sdl::launch_pdl(wsum_kernel<T>, dim3(ndc, rows), dim3(kGroup), 0, st, A, none, V, temp,
                            (const float2*)w.rowstat, ndc, 0, 0, (const int*)nullptr, w.wsum);
    if (e == cudaSuccess)
        e = sdl::launch_pdl(finish_kernel<T>, dim3(rows), dim3(1024), 0, st, A, none, V, temp, (const float2*)w.rowstat,
                            ndc, 0, 0, (const int*)nullptr, (const int*)nullptr, uniforms, nu, u_base, u_off,
                            (const uint64_t*)w.wsum, w.wsum_p, (const int*)nullptr, out,
                            (int*)nullptr, err);
    if (e != cudaSuccess) return sdl::fail(SDL_ERR_CUDA, cudaGetErrorString(e));
    return sdl::check_launch("sample_logits");
}

FusedWs carve_fused(void* base, int B, int gamma, int nchunks, int ndc, size_t* bytes) {
    FusedWs w;
    char* p = static_cast<char*>(base);
    const int R = 2 * gamma + 1;
    size_t o = 0;
    w.ctrl = reinterpret_cast<int*>(p);
    o = kCtrlBytes;
    w.stats = reinterpret_cast<float2*>(p + o);
    o = align256(o + (size_t)B * R * nchunks * sizeof(float2));
    w.rowstat = reinterpret_cast<float2*>(p + o);
    o = align256(o + (size_t)B * R * sizeof(float2));
    w.acc = reinterpret_cast<double*>(p + o);
    o = align256(o + (size_t)B * gamma * sizeof(double));
    w.wsum = reinterpret_cast<uint64_t*>(p + o);
    o = align256(o + (size_t)B * ndc * sizeof(uint64_t));
    w.wsum_p = reinterpret_cast<uint64_t*>(p + o);
    o = align256(o + (size_t)B * ndc * sizeof(uint64_t));
    if (bytes) *bytes = o;
    return w;
}

size_t fused_walk_smem(int B, int gamma) {
    return (size_t)B * gamma * sizeof(double) + (size_t)B * (gamma + 1) * sizeof(float);
}

// 0 (default): the five-launch chain; 1: the one-launch kernel where it
// applies.  Measured on B200 at C3 (32 sequences, gamma 5, vocab 151,936,
// fp32 logits): 76 us for the one-launch kernel against 63 us for the
// chain, whose statistics launch spreads 6,688 CTAs over every SM while
// the clusters hold 1-2 CTAs per SM and serialise their phases.
int g_sampler_mode = 0;

// Clusters of `cs` CTAs of spec_fused_kernel<T> resident at once with
// `smem` bytes of dynamic shared memory (0 when the query fails).
template <typename T>
int fused_active_clusters(int cs, size_t smem) {
    static std::mutex mu;
    static std::map<std::pair<int, size_t>, int> cache;
    std::lock_guard<std::mutex> lock(mu);
    const auto key = std::make_pair(cs, smem);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(cs, 1, 1);
    cfg.blockDim = dim3(kFuseThreads);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = cs;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, spec_fused_kernel<T>, &cfg) != cudaSuccess) {
        (void)cudaGetLastError();
        n = 0;
    }
    cache[key] = n;
    return n;
}

// Launches the fused kernel when it applies (returns 1), else returns 0
// and launches nothing; a negative value is an error status.
template <typename T>
int spec_fused_try(const T* pl, int64_t p_sb, int64_t p_sj, const T* ql, int64_t q_sb, int64_t q_sj, float temp,
                   const int* prop, int B, int gamma, int V, const float* uniforms, int64_t nu, int64_t* u_base,
                   int64_t u_skip, int* tokens, int* n_out, void* ws_base, size_t ws_bytes, int* err,
                   cudaStream_t st) {
    if (g_sampler_mode != 1) return 0;
    const int nchunks = (V + kChunk - 1) / kChunk;
    const int ndc = (V + kDrawChunk - 1) / kDrawChunk;
    if (B > kMaxFusedSeqs || ndc > kFuseMaxDrawChunks || 2 * gamma + 1 > kMaxFusedRows) return 0;
    size_t need = 0;
    (void)carve_fused(nullptr, B, gamma, nchunks, ndc, &need);
    if (need > ws_bytes) return 0;
    const size_t smem = fused_walk_smem(B, gamma);
    if (smem > 200 * 1024) return 0;
    static std::mutex mu;
    static size_t configured = 0;
    {
        std::lock_guard<std::mutex> lock(mu);
        if (smem > 48 * 1024 && smem > configured) {
            if (cudaFuncSetAttribute(spec_fused_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
                cudaSuccess) {
                (void)cudaGetLastError();
                return 0;
            }
            configured = smem;
        }
    }
    // the largest cluster whose grid is resident at once (the look-back wait
    // of step 2 needs every lower-numbered sequence running or done)
    int cs = kFuseCluster;
    while (cs >= 1 && fused_active_clusters<T>(cs, smem) < B) cs /= 2;
    if (cs < 1) return 0;
    FusedWs w = carve_fused(ws_base, B, gamma, nchunks, ndc, nullptr);
    Rows<T> A{pl, p_sb, p_sj, gamma + 1, B * (gamma + 1)};
    Rows<T> Q{ql, q_sb, q_sj, gamma, B * gamma};
    cudaError_t e = sdl::launch_pdl_cluster(spec_fused_kernel<T>, dim3(cs, B), dim3(kFuseThreads), smem, st,
                                            (unsigned)cs, A, Q, V, temp, prop, B, gamma, uniforms, nu, u_base, u_skip,
                                            tokens, n_out, w, nchunks, ndc, err);
    if (e != cudaSuccess) return -sdl::fail(SDL_ERR_CUDA, cudaGetErrorString(e));
    const int rc = sdl::check_launch("spec_fused_kernel");
    return rc == SDL_OK ? 1 : -rc;
}

template <typename T>
int spec_logits_t(const T* pl, int64_t p_sb, int64_t p_sj, const T* ql, int64_t q_sb, int64_t q_sj, float temp,
                  const int* prop, int B, int gamma, int V, const float* uniforms, int64_t nu, int64_t* u_base,
                  int64_t u_skip, int* tokens, int* n_out, void* ws_base, size_t ws_bytes, int* err,
                  const int* n_valid, cudaStream_t st) {
    // a device sequence count (padded captured batches) takes the chain
    const int fused = n_valid != nullptr ? 0
                                         : spec_fused_try<T>(pl, p_sb, p_sj, ql, q_sb, q_sj, temp, prop, B, gamma, V,
                                                             uniforms, nu, u_base, u_skip, tokens, n_out, ws_base,
                                                             ws_bytes, err, st);
    if (fused != 0) return fused > 0 ? SDL_OK : -fused;
    const int nchunks = (V + kChunk - 1) / kChunk;
    const int ndc = (V + kDrawChunk - 1) / kDrawChunk;
    const int prow = B * (gamma + 1), qrow = B * gamma;
    Ws w = carve(ws_base, prow + qrow, B, nchunks, ndc);
    Rows<T> A{pl, p_sb, p_sj, gamma + 1, prow};
    Rows<T> Q{ql, q_sb, q_sj, gamma, qrow};
    const size_t smem = (size_t)B * gamma * sizeof(double) + (size_t)B * (gamma + 1) * sizeof(float);
    static size_t configured = 0;
    if (smem > 48 * 1024 && smem > configured) {
        cudaError_t e = cudaFuncSetAttribute(accept_logits_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)smem);
        if (e != cudaSuccess) return sdl::fail(SDL_ERR_CUDA, cudaGetErrorString(e));
        configured = smem;
    }
    cudaError_t e = sdl::launch_pdl(stats_kernel<T>, dim3(nchunks, prow + qrow), dim3(kGroup), 0, st, A, Q, V, temp,
                                    w.stats);
    if (e == cudaSuccess)
        e = sdl::launch_pdl(merge_kernel, dim3(prow + qrow), dim3(128), 0, st, (const float2*)w.stats, nchunks,
                            w.rowstat);
    if (e == cudaSuccess)
        e = sdl::launch_pdl(accept_logits_kernel<T>, dim3(1), dim3(1024), smem, st, A, Q, V, temp,
                            (const float2*)w.rowstat, prop, B, gamma, uniforms, nu, u_base, u_skip, w.n_acc, w.u_bits,
                            err, n_valid);
    if (e == cudaSuccess)
        e = sdl::launch_pdl(wsum_kernel<T>, dim3(ndc, B), dim3(kGroup), 0, st, A, Q, V, temp,
                            (const float2*)w.rowstat, ndc, 1, gamma, (const int*)w.n_acc, w.wsum);
    if (e == cudaSuccess)
        e = sdl::launch_pdl(finish_kernel<T>, dim3(B), dim3(1024), 0, st, A, Q, V, temp, (const float2*)w.rowstat,
                            ndc, 1, gamma, (const int*)w.n_acc, (const int*)w.u_bits, uniforms, nu,
                            (const int64_t*)nullptr, (int64_t)0, (const uint64_t*)w.wsum, w.wsum_p,
                            prop, tokens, n_out, err);
    if (e != cudaSuccess) return sdl::fail(SDL_ERR_CUDA, cudaGetErrorString(e));
    return sdl::check_launch("spec_sample_logits");
}

}  // namespace

// Canonical p = softmax(logits / T) rows (one CTA per row); used by
// sdl_logits_to_probs for temperature sampling.
int sdl_probs_canon(const void* logits, int32_t dtype, int64_t row_stride, int32_t rows, int32_t vocab, float temp,
                    float* probs, int64_t probs_stride, cudaStream_t st) {
    if ((vocab + kChunk - 1) / kChunk > kMaxChunks) return sdl::fail(SDL_ERR_UNSUPPORTED, "vocab above 8M");
    if (dtype == SDL_F32)
        probs_canon_kernel<float><<<rows, 1024, 0, st>>>((const float*)logits, row_stride, vocab, temp, probs,
                                                         probs_stride);
    else if (dtype == SDL_BF16)
        probs_canon_kernel<__nv_bfloat16><<<rows, 1024, 0, st>>>((const __nv_bfloat16*)logits, row_stride, vocab, temp,
                                                                 probs, probs_stride);
    else if (dtype == SDL_F16)
        probs_canon_kernel<__half><<<rows, 1024, 0, st>>>((const __half*)logits, row_stride, vocab, temp, probs,
                                                          probs_stride);
    else
        return sdl::fail(SDL_ERR_UNSUPPORTED, "sdl_logits_to_probs: dtype");
    return sdl::check_launch("probs_canon_kernel");
}

extern "C" size_t sdl_sampler_workspace_bytes(int32_t rows, int32_t vocab) {
    if (rows < 0 || vocab < 1) return 0;
    const int nchunks = (vocab + kChunk - 1) / kChunk;
    const int ndc = (vocab + kDrawChunk - 1) / kDrawChunk;
    // statistics for `rows` logit rows and draw sums for as many draws
    return carve(nullptr, rows, rows, nchunks, ndc).bytes;
}

extern "C" int sdl_sample_logits_rows(const void* logits, int32_t dtype, int64_t row_stride, int32_t rows,
                                      int32_t vocab, float temperature, float eps, const float* uniforms,
                                      int64_t num_uniforms, const int64_t* u_base, int64_t u_offset, int32_t* out,
                                      void* workspace, size_t workspace_bytes, int32_t* err, void* stream) {
    if (!logits || !uniforms || !out || rows < 0 || vocab < 1 || row_stride < vocab)
        return sdl::fail(SDL_ERR_INVALID, "sdl_sample_logits_rows: bad args");
    if (rows == 0) return SDL_OK;
    const int nchunks = (vocab + kChunk - 1) / kChunk;
    const int ndc = (vocab + kDrawChunk - 1) / kDrawChunk;
    if (ndc > kMaxDrawChunks) return sdl::fail(SDL_ERR_UNSUPPORTED, "sdl_sample_logits_rows: vocab above 2M");
    if (rows > 65535) return sdl::fail(SDL_ERR_UNSUPPORTED, "sdl_sample_logits_rows: more than 65535 rows");
    if (!workspace || workspace_bytes < carve(nullptr, rows, rows, nchunks, ndc).bytes ||
        reinterpret_cast<uintptr_t>(workspace) % 256)
        return sdl::fail(SDL_ERR_WORKSPACE, "sdl_sample_logits_rows: workspace missing, small or not 256-B aligned");
    const float t = temperature > eps ? temperature : eps;
    cudaStream_t st = sdl::as_stream(stream);
    if (dtype == SDL_F32)
        return sample_logits_t<float>((const float*)logits, row_stride, rows, vocab, t, uniforms, num_uniforms, u_base,
                                      u_offset, out, workspace, err, st);
    if (dtype == SDL_BF16)
        return sample_logits_t<__nv_bfloat16>((const __nv_bfloat16*)logits, row_stride, rows, vocab, t, uniforms,
                                              num_uniforms, u_base, u_offset, out, workspace, err, st);
    if (dtype == SDL_F16)
        return sample_logits_t<__half>((const __half*)logits, row_stride, rows, vocab, t, uniforms, num_uniforms,
                                       u_base, u_offset, out, workspace, err, st);
    return sdl::fail(SDL_ERR_UNSUPPORTED, "sdl_sample_logits_rows: dtype");
}

namespace {
int spec_sample_logits_impl(const void* p_logits, int64_t p_sb, int64_t p_sj, const void* q_logits, int64_t q_sb,
                            int64_t q_sj, int32_t dtype, float temperature, float eps, const int32_t* proposals,
                            int32_t B, int32_t gamma, int32_t vocab, const float* uniforms, int64_t num_uniforms,
                            int64_t* u_base, int64_t u_skip, int32_t* tokens, int32_t* n_out, void* workspace,
                            size_t workspace_bytes, int32_t* err, const int32_t* n_valid, void* stream) {
    if (!p_logits || !q_logits || !proposals || !uniforms || !tokens || !n_out || B < 0 || gamma < 1 || gamma > 32 ||
        vocab < 1)
        return sdl::fail(SDL_ERR_INVALID, "sdl_spec_sample_logits: bad args (gamma must be 1..32)");
    if (B == 0) return SDL_OK;
    const int nchunks = (vocab + kChunk - 1) / kChunk;
    const int ndc = (vocab + kDrawChunk - 1) / kDrawChunk;
    if (ndc > kMaxDrawChunks) return sdl::fail(SDL_ERR_UNSUPPORTED, "sdl_spec_sample_logits: vocab above 2M");
    const int stat_rows = B * (2 * gamma + 1);
    if (stat_rows > 65535) return sdl::fail(SDL_ERR_UNSUPPORTED, "sdl_spec_sample_logits: too many rows");
    if (!workspace || workspace_bytes < carve(nullptr, stat_rows, B, nchunks, ndc).bytes ||
        reinterpret_cast<uintptr_t>(workspace) % 256)
        return sdl::fail(SDL_ERR_WORKSPACE, "sdl_spec_sample_logits: workspace missing, small or not 256-B aligned");
    const size_t smem = (size_t)B * gamma * sizeof(double) + (size_t)B * (gamma + 1) * sizeof(float);
    if (smem > 200 * 1024) return sdl::fail(SDL_ERR_INVALID, "sdl_spec_sample_logits: batch too large for one CTA");
    const float t = temperature > eps ? temperature : eps;
    cudaStream_t st = sdl::as_stream(stream);
    if (dtype == SDL_F32)
        return spec_logits_t<float>((const float*)p_logits, p_sb, p_sj, (const float*)q_logits, q_sb, q_sj, t,
                                    proposals, B, gamma, vocab, uniforms, num_uniforms, u_base, u_skip, tokens, n_out,
                                    workspace, workspace_bytes, err, n_valid, st);
    if (dtype == SDL_BF16)
        return spec_logits_t<__nv_bfloat16>((const __nv_bfloat16*)p_logits, p_sb, p_sj,
                                            (const __nv_bfloat16*)q_logits, q_sb, q_sj, t, proposals, B, gamma, vocab,
                                            uniforms, num_uniforms, u_base, u_skip, tokens, n_out, workspace,
                                            workspace_bytes, err, n_valid, st);
    if (dtype == SDL_F16)
        return spec_logits_t<__half>((const __half*)p_logits, p_sb, p_sj, (const __half*)q_logits, q_sb, q_sj, t,
                                     proposals, B, gamma, vocab, uniforms, num_uniforms, u_base, u_skip, tokens,
                                     n_out, workspace, workspace_bytes, err, n_valid, st);
    return sdl::fail(SDL_ERR_UNSUPPORTED, "sdl_spec_sample_logits: dtype");
}
}  // namespace

extern "C" int sdl_spec_sample_logits(const void* p_logits, int64_t p_sb, int64_t p_sj, const void* q_logits,
                                      int64_t q_sb, int64_t q_sj, int32_t dtype, float temperature, float eps,
                                      const int32_t* proposals, int32_t B, int32_t gamma, int32_t vocab,
                                      const float* uniforms, int64_t num_uniforms, int64_t* u_base, int64_t u_skip,
                                      int32_t* tokens, int32_t* n_out, void* workspace, size_t workspace_bytes,
                                      int32_t* err, void* stream) {
    return spec_sample_logits_impl(p_logits, p_sb, p_sj, q_logits, q_sb, q_sj, dtype, temperature, eps, proposals, B,
                                   gamma, vocab, uniforms, num_uniforms, u_base, u_skip, tokens, n_out, workspace,
                                   workspace_bytes, err, nullptr, stream);
}

extern "C" int sdl_spec_sample_logits_n(const void* p_logits, int64_t p_sb, int64_t p_sj, const void* q_logits,
                                        int64_t q_sb, int64_t q_sj, int32_t dtype, float temperature, float eps,
                                        const int32_t* proposals, int32_t B, int32_t gamma, int32_t vocab,
                                        const float* uniforms, int64_t num_uniforms, int64_t* u_base, int64_t u_skip,
                                        int32_t* tokens, int32_t* n_out, void* workspace, size_t workspace_bytes,
                                        int32_t* err, const int32_t* n_valid, void* stream) {
    if (!n_valid) return sdl::fail(SDL_ERR_INVALID, "sdl_spec_sample_logits_n: n_valid is NULL");
    return spec_sample_logits_impl(p_logits, p_sb, p_sj, q_logits, q_sb, q_sj, dtype, temperature, eps, proposals, B,
                                   gamma, vocab, uniforms, num_uniforms, u_base, u_skip, tokens, n_out, workspace,
                                   workspace_bytes, err, n_valid, stream);
}

extern "C" int sdl_set_spec_sampler_mode(int32_t mode) {
    if (mode != 0 && mode != 1) return sdl::fail(SDL_ERR_INVALID, "sdl_set_spec_sampler_mode: mode must be 0 or 1");
    g_sampler_mode = mode;
    return SDL_OK;
}
