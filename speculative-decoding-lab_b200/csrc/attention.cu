// Paged attention for decode, verify (extend) and prefill rows.
//
// Semantics (one definition for all three reference entry points):
// query row j of batch entry b sits at absolute position starts[b] + j and
// attends key positions [0, starts[b] + j] of that sequence's pages,
// softmax-scaled by `scale`, with q head h reading kv head h / (Hq/Hkv).
//   paged_attention_decode  engine/attention.py:96-118  (chunk 1, start = len-1)
//   paged_attention_extend  engine/attention.py:170-215 (causal offset mask :204-208)
//   paged_attention_prefill_chunk engine/attention.py:121-167 (start 0, dense K/V)
//
// Two implementations:
//  * attn_tc_kernel  (bf16/f16, head_dim 64/128, block_size 16): a split-K
//    flash-decoding kernel.  One producer warp streams pages with TMA
//    (cp.async.bulk.tensor, 128B swizzle, one 2 KB box per kv head and 64
//    columns) through a 4-stage mbarrier ring; consumer warps compute
//    S^T = K_page * Q^T and O^T += V_page^T * P^T with mma.sync m16n8k16
//    (tokens on the M side so GQA query rows fill the N side), online softmax
//    in the log2 domain with warp-shuffle column reductions, and P carried
//    as a hi+lo pair of 16-bit values so the PV product keeps ~16 mantissa
//    bits.  Splits write fp32 partials; attn_combine_kernel merges them.
//  * attn_generic_kernel (any dtype, any head_dim <= 256, any block size):
//    one warp per query row on CUDA cores, fp32 arithmetic with expf; used
//    for fp32 pools and shapes the tensor-core kernel does not cover.
#include "sdl_common.cuh"

#include <cuda.h>
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>

namespace {

constexpr int kPage = 16;          // tokens per TMA page (= block_size on the TC path)
constexpr int kStages = 4;         // TMA ring depth
constexpr int kMaxConsumerWarps = 8;
constexpr int kBoxBytes = kPage * 128;  // one [16 tokens][64 cols] 16-bit box
constexpr uint32_t kWaitLimit = 1u << 20;

struct TcParams {
    const void* q;
    int64_t q_sb, q_sj, q_sh;
    void* out;
    int64_t o_sb, o_sj, o_sh;
    int out_dtype;
    const int32_t* table;
    int width, capacity, layer;
    const int32_t* rows;
    const int32_t* starts;
    const int32_t* valid_rows;
    int dense, kv_len;
    int B, chunk, Hq, Hkv, ratio;
    int pps, nsplit;
    int g_cta, wpg, ncoltiles;
    int stage_bytes;
    float scale_log2;
    float* o_part;
    float* ml_part;
    int32_t* err;
};

SDL_DEV uint32_t ld_u32(const void* p) { return *reinterpret_cast<const uint32_t*>(p); }

template <int HD, int NTG, typename T>
__global__ void __launch_bounds__((kMaxConsumerWarps + 1) * 32)
attn_tc_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv, const TcParams p) {
    constexpr int DO = HD / 64;
    constexpr int KSTEPS = HD / 16;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * p.stage_bytes);
    uint64_t* empty = full + kStages;
    __shared__ int s_abort_flag;
    volatile int* s_abort = &s_abort_flag;

    // Launched as a programmatic dependent: everything below may read what
    // the preceding kernel (K/V append, block-table reserve) wrote.
    pdl_wait();

    const int b = blockIdx.z;
    const int split = blockIdx.x;
    const int coltile = blockIdx.y % p.ncoltiles;
    const int kvgrp = blockIdx.y / p.ncoltiles;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ncons = p.g_cta * p.wpg;

    const int start = p.starts[b];
    const int nvalid = p.valid_rows ? min(p.valid_rows[b], p.chunk) : p.chunk;
    const int ncol = p.chunk * p.ratio;
    const int tile_cols = p.wpg * NTG * 8;
    const int col0 = coltile * tile_cols;
    if (col0 >= ncol || col0 / p.ratio >= nvalid) return;
    const int col_last = min(col0 + tile_cols, ncol) - 1;
    const int j_last = min(col_last / p.ratio, nvalid - 1);
    const int lmax = start + j_last + 1;
    const int npages = (lmax + kPage - 1) / kPage;
    const int pbeg = split * p.pps;
    const int pend = min(npages, pbeg + p.pps);
    if (lmax <= 0 || pbeg >= pend) return;
    const int np = pend - pbeg;
    const int row = p.dense ? 0 : p.rows[b];

    if (threadIdx.x == 0) {
        *s_abort = 0;
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], ncons);
        }
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == ncons) {
        // ------------------------------------------------------- producer
        if (lane == 0) { prefetch_tmap(&tmk); prefetch_tmap(&tmv); }
        int issued = 0;
        bool stop = false;
        for (int i0 = 0; i0 < np && !stop; i0 += 32) {
            int tok0 = 0;
            if (i0 + lane < np) {
                int pg = pbeg + i0 + lane;
                if (p.dense) {
                    tok0 = b * p.kv_len + pg * kPage;
                } else {
                    int phys = pg < p.width ? p.table[(int64_t)row * p.width + pg] : -1;
                    if (phys < 0 || phys >= p.capacity) { sdl_raise(p.err, SDL_DEVERR_BAD_INDEX); phys = 0; }
                    tok0 = (p.layer * p.capacity + phys) * kPage;
                }
            }
            const int cnt = min(32, np - i0);
            for (int k = 0; k < cnt; ++k) {
                const int t0 = __shfl_sync(0xffffffffu, tok0, k);
                const int i = i0 + k;
                const int st = i % kStages;
                if (i >= kStages) {
                    int ok = 1;
                    if (lane == 0) ok = mbar_wait_bounded(&empty[st], ((i / kStages) - 1) & 1, kWaitLimit) ? 1 : 0;
                    ok = __shfl_sync(0xffffffffu, ok, 0);
                    if (!ok || *s_abort) {
                        if (lane == 0 && !ok) { sdl_raise(p.err, SDL_DEVERR_TIMEOUT); *s_abort = 1; }
                        stop = true;
                        break;
                    }
                }
                if (lane == 0) {
                    mbar_arrive_expect_tx(&full[st], p.stage_bytes);
                    uint8_t* sbuf = smem + st * p.stage_bytes;
                    for (int gi = 0; gi < p.g_cta; ++gi) {
                        const int g = kvgrp * p.g_cta + gi;
                        uint8_t* kb = sbuf + gi * (2 * DO * kBoxBytes);
#pragma unroll
                        for (int dd = 0; dd < DO; ++dd) {
                            tma_load_4d(kb + dd * kBoxBytes, &tmk, &full[st], 0, dd, g, t0);
                            tma_load_4d(kb + (DO + dd) * kBoxBytes, &tmv, &full[st], 0, dd, g, t0);
                        }
                    }
                }
                __syncwarp();
                issued = i + 1;
            }
        }
        __syncthreads();
        // Drain: never leave the CTA with bulk copies still landing in smem.
        if (lane == 0 && *s_abort) {
            for (int i = max(0, issued - kStages); i < issued; ++i)
                (void)mbar_wait_bounded(&full[i % kStages], (i / kStages) & 1, kWaitLimit);
        }
        pdl_launch_dependents();
        return;
    }

    // ----------------------------------------------------------- consumers
    const int gi = warp / p.wpg, wc = warp % p.wpg;
    const int g = kvgrp * p.g_cta + gi;
    const int cbase = col0 + wc * NTG * 8;
    const int tq = lane & 3, grp = lane >> 2;

    uint32_t qf[KSTEPS][NTG][2];
#pragma unroll
    for (int nt = 0; nt < NTG; ++nt) {
        const int col = cbase + nt * 8 + grp;
        const bool ok = col < ncol && col / p.ratio < nvalid;
        const T* qp = nullptr;
        if (ok) {
            const int j = col / p.ratio, h = g * p.ratio + col % p.ratio;
            qp = reinterpret_cast<const T*>(p.q) + b * p.q_sb + j * p.q_sj + h * p.q_sh;
        }
#pragma unroll
        for (int ks = 0; ks < KSTEPS; ++ks) {
            qf[ks][nt][0] = ok ? ld_u32(qp + ks * 16 + 2 * tq) : 0u;
            qf[ks][nt][1] = ok ? ld_u32(qp + ks * 16 + 8 + 2 * tq) : 0u;
        }
    }
    int lim[NTG][2];
    float m_run[NTG][2], l_run[NTG][2];
#pragma unroll
    for (int nt = 0; nt < NTG; ++nt)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            const int col = cbase + nt * 8 + 2 * tq + e;
            const int j = col / p.ratio;
            lim[nt][e] = (col < ncol && j < nvalid) ? start + j + 1 : lmax;
            m_run[nt][e] = -INFINITY;
            l_run[nt][e] = 0.f;
        }
    float acc[KSTEPS][NTG][4];
#pragma unroll
    for (int mt = 0; mt < KSTEPS; ++mt)
#pragma unroll
        for (int nt = 0; nt < NTG; ++nt)
#pragma unroll
            for (int r = 0; r < 4; ++r) acc[mt][nt][r] = 0.f;

    const uint32_t sbase = smem_u32(smem);
    const int mi = lane >> 3, mr = lane & 7;
    bool aborted = false;
    for (int i = 0; i < np; ++i) {
        const int st = i % kStages;
        const bool ok = __all_sync(0xffffffffu, mbar_wait_bounded(&full[st], (i / kStages) & 1, kWaitLimit));
        if (!ok) {
            if (lane == 0) { sdl_raise(p.err, SDL_DEVERR_TIMEOUT); *s_abort = 1; }
            aborted = true;
            break;
        }
        const uint32_t kbase = sbase + st * p.stage_bytes + gi * (2 * DO * kBoxBytes);
        const uint32_t vbase = kbase + DO * kBoxBytes;

        // S^T[t][col] = sum_d K[t][d] Q[col][d]
        float s[NTG][4];
#pragma unroll
        for (int nt = 0; nt < NTG; ++nt)
#pragma unroll
            for (int r = 0; r < 4; ++r) s[nt][r] = 0.f;
#pragma unroll
        for (int ks = 0; ks < KSTEPS; ++ks) {
            const int t = mr + ((mi & 1) << 3);
            const int dd = ks * 16 + ((mi >> 1) << 3);
            const uint32_t addr = kbase + (dd >> 6) * kBoxBytes + t * 128 + ((((dd & 63) >> 3) ^ (t & 7)) << 4);
            uint32_t a[4];
            ldmatrix_x4(addr, a[0], a[1], a[2], a[3]);
#pragma unroll
            for (int nt = 0; nt < NTG; ++nt) mma_16816<T>(s[nt], a, qf[ks][nt][0], qf[ks][nt][1]);
        }

        // Online softmax per query column (log2 domain).
        const int pos_lo = (pbeg + i) * kPage + grp, pos_hi = pos_lo + 8;
        uint32_t pb[NTG][2], pl[NTG][2];
#pragma unroll
        for (int nt = 0; nt < NTG; ++nt) {
            float pv[4];
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const float x0 = pos_lo < lim[nt][e] ? s[nt][e] * p.scale_log2 : -INFINITY;
                const float x1 = pos_hi < lim[nt][e] ? s[nt][2 + e] * p.scale_log2 : -INFINITY;
                float mx = fmaxf(x0, x1);
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
                const float mnew = fmaxf(m_run[nt][e], mx);
                const float muse = mnew == -INFINITY ? 0.f : mnew;
                const float alpha = exp2f(m_run[nt][e] - muse);
                const float p0 = exp2f(x0 - muse), p1 = exp2f(x1 - muse);
                l_run[nt][e] = l_run[nt][e] * alpha + p0 + p1;
                m_run[nt][e] = mnew;
#pragma unroll
                for (int mt = 0; mt < KSTEPS; ++mt) {
                    acc[mt][nt][e] *= alpha;
                    acc[mt][nt][2 + e] *= alpha;
                }
                pv[e] = p0;
                pv[2 + e] = p1;
            }
            const float h0 = round_trip<T>(pv[0]), h1 = round_trip<T>(pv[1]);
            const float h2 = round_trip<T>(pv[2]), h3 = round_trip<T>(pv[3]);
            pb[nt][0] = movmatrix_trans(pack2<T>(pv[0], pv[1]));
            pb[nt][1] = movmatrix_trans(pack2<T>(pv[2], pv[3]));
            pl[nt][0] = movmatrix_trans(pack2<T>(pv[0] - h0, pv[1] - h1));
            pl[nt][1] = movmatrix_trans(pack2<T>(pv[2] - h2, pv[3] - h3));
        }

        // O^T[d][col] += sum_t V[t][d] P^T[t][col]
#pragma unroll
        for (int mt = 0; mt < KSTEPS; ++mt) {
            const int t = mr + ((mi >> 1) << 3);
            const int dd = mt * 16 + ((mi & 1) << 3);
            const uint32_t addr = vbase + (dd >> 6) * kBoxBytes + t * 128 + ((((dd & 63) >> 3) ^ (t & 7)) << 4);
            uint32_t a[4];
            ldmatrix_x4_trans(addr, a[0], a[1], a[2], a[3]);
#pragma unroll
            for (int nt = 0; nt < NTG; ++nt) {
                mma_16816<T>(acc[mt][nt], a, pb[nt][0], pb[nt][1]);
                mma_16816<T>(acc[mt][nt], a, pl[nt][0], pl[nt][1]);
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[st]);
    }
    __syncthreads();
    pdl_launch_dependents();  // the split merge may be scheduled during the epilogue
    if (aborted || *s_abort) return;

    // Epilogue: finished rows write the output, split rows write partials.
#pragma unroll
    for (int nt = 0; nt < NTG; ++nt)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            float l = l_run[nt][e];
            l += __shfl_xor_sync(0xffffffffu, l, 4);
            l += __shfl_xor_sync(0xffffffffu, l, 8);
            l += __shfl_xor_sync(0xffffffffu, l, 16);
            const int col = cbase + nt * 8 + 2 * tq + e;
            if (col >= ncol) continue;
            const int j = col / p.ratio;
            if (j >= nvalid) continue;
            const int h = g * p.ratio + col % p.ratio;
            const int L = start + j + 1;
            const int np_c = (L + kPage - 1) / kPage;
            if (pbeg >= np_c) continue;
            const int ns_c = (np_c + p.pps - 1) / p.pps;
            if (ns_c == 1) {
                const float inv = 1.f / l;
                const int64_t ob = b * p.o_sb + j * p.o_sj + h * p.o_sh;
#pragma unroll
                for (int mt = 0; mt < KSTEPS; ++mt) {
                    store_from_f32(p.out, ob + mt * 16 + grp, p.out_dtype, acc[mt][nt][e] * inv);
                    store_from_f32(p.out, ob + mt * 16 + grp + 8, p.out_dtype, acc[mt][nt][2 + e] * inv);
                }
            } else {
                const int64_t idx = (((int64_t)b * p.nsplit + split) * p.chunk + j) * p.Hq + h;
                float* op = p.o_part + idx * HD;
#pragma unroll
                for (int mt = 0; mt < KSTEPS; ++mt) {
                    op[mt * 16 + grp] = acc[mt][nt][e];
                    op[mt * 16 + grp + 8] = acc[mt][nt][2 + e];
                }
                if (grp == 0) {
                    p.ml_part[idx * 2] = m_run[nt][e];
                    p.ml_part[idx * 2 + 1] = l;
                }
            }
        }
}

// Merge split-K partials (m in log2 units, unnormalised O, l).  One warp per
// (sequence, chunk row, q head): lanes reduce the split maxima and
// denominators in parallel, then each lane owns 4 consecutive head dims and
// keeps 8 splits' loads in flight at once (the merge is latency bound).
__global__ void __launch_bounds__(128) attn_combine_kernel(TcParams p, int hd) {
    pdl_wait();  // partials come from the attention launch just before
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r = blockIdx.x * 4 + warp;
    if (r >= p.B * p.chunk * p.Hq) return;
    const int h = r % p.Hq;
    const int j = (r / p.Hq) % p.chunk;
    const int b = r / (p.Hq * p.chunk);
    const int nvalid = p.valid_rows ? min(p.valid_rows[b], p.chunk) : p.chunk;
    if (j >= nvalid) return;
    const int L = p.starts[b] + j + 1;
    if (L <= 0) return;
    const int np_c = (L + kPage - 1) / kPage;
    const int ns = (np_c + p.pps - 1) / p.pps;
    if (ns <= 1) return;
    const int64_t idx0 = (((int64_t)b * p.nsplit) * p.chunk + j) * p.Hq + h;
    const int64_t sstride = (int64_t)p.chunk * p.Hq;
    float M = -INFINITY;
    for (int s = lane; s < ns; s += 32) M = fmaxf(M, p.ml_part[(idx0 + s * sstride) * 2]);
    M = warp_max(M);
    float den = 0.f;
    for (int s = lane; s < ns; s += 32) {
        const float* ml = p.ml_part + (idx0 + s * sstride) * 2;
        den += exp2f(ml[0] - M) * ml[1];
    }
    den = warp_sum(den);
    const float inv = 1.f / den;
    const int64_t ob = b * p.o_sb + j * p.o_sj + h * p.o_sh;
    for (int d0 = lane * 4; d0 < hd; d0 += 128) {
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        int s = 0;
        for (; s + 8 <= ns; s += 8) {
            float w[8];
            float4 o[8];
#pragma unroll
            for (int t = 0; t < 8; ++t) {
                const int64_t idx = idx0 + (s + t) * sstride;
                w[t] = p.ml_part[idx * 2];
                o[t] = *reinterpret_cast<const float4*>(p.o_part + idx * hd + d0);
            }
#pragma unroll
            for (int t = 0; t < 8; ++t) {
                const float wt = exp2f(w[t] - M);
                acc.x += wt * o[t].x;
                acc.y += wt * o[t].y;
                acc.z += wt * o[t].z;
                acc.w += wt * o[t].w;
            }
        }
        for (; s < ns; ++s) {
            const int64_t idx = idx0 + s * sstride;
            const float wt = exp2f(p.ml_part[idx * 2] - M);
            const float4 o = *reinterpret_cast<const float4*>(p.o_part + idx * hd + d0);
            acc.x += wt * o.x;
            acc.y += wt * o.y;
            acc.z += wt * o.z;
            acc.w += wt * o.w;
        }
        store_from_f32(p.out, ob + d0, p.out_dtype, acc.x * inv);
        store_from_f32(p.out, ob + d0 + 1, p.out_dtype, acc.y * inv);
        store_from_f32(p.out, ob + d0 + 2, p.out_dtype, acc.z * inv);
        store_from_f32(p.out, ob + d0 + 3, p.out_dtype, acc.w * inv);
    }
}

// ------------------------------------------------------------ generic path
struct GenParams {
    const void* q;
    int64_t q_sb, q_sj, q_sh;
    void* out;
    int64_t o_sb, o_sj, o_sh;
    int out_dtype;
    const void* k;  // paged pool or dense tensor
    const void* v;
    const int32_t* table;
    int width, capacity, layer, bs;
    const int32_t* rows;
    const int32_t* starts;
    const int32_t* valid_rows;
    int dense, kv_len;
    int B, chunk, Hq, Hkv, ratio, hd;
    float scale;
    int32_t* err;
};

template <typename T>
SDL_DEV const T* gen_row(const GenParams& p, const T* base, int b, int row, int t, int g) {
    int64_t r;
    if (p.dense) {
        r = (int64_t)b * p.kv_len + t;
    } else {
        const int bi = t / p.bs;
        int phys = bi < p.width ? p.table[(int64_t)row * p.width + bi] : -1;
        if (phys < 0 || phys >= p.capacity) { sdl_raise(p.err, SDL_DEVERR_BAD_INDEX); phys = 0; }
        r = ((int64_t)p.layer * p.capacity + phys) * p.bs + t % p.bs;
    }
    return base + (r * p.Hkv + g) * p.hd;
}

template <typename T>
__global__ void __launch_bounds__(128) attn_generic_kernel(const GenParams p) {
    __shared__ float qs[4][256];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r = blockIdx.x * 4 + warp;
    const int b = blockIdx.y;
    const int j = r / p.Hq, h = r % p.Hq;
    if (j >= p.chunk) return;
    const int nvalid = p.valid_rows ? min(p.valid_rows[b], p.chunk) : p.chunk;
    if (j >= nvalid) return;
    const int g = h / p.ratio;
    const int L = p.starts[b] + j + 1;
    const int row = p.dense ? 0 : p.rows[b];
    const T* qp = reinterpret_cast<const T*>(p.q) + b * p.q_sb + j * p.q_sj + h * p.q_sh;
    for (int d = lane; d < p.hd; d += 32) qs[warp][d] = to_f32<T>(qp[d]);
    __syncwarp();
    const T* kb = reinterpret_cast<const T*>(p.k);
    const T* vb = reinterpret_cast<const T*>(p.v);
    float acc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = 0.f;
    float m = -INFINITY, l = 0.f;
    for (int t0 = 0; t0 < L; t0 += 32) {
        const int t = t0 + lane;
        float s = -INFINITY;
        if (t < L) {
            const T* kr = gen_row<T>(p, kb, b, row, t, g);
            float dot = 0.f;
            for (int d = 0; d < p.hd; ++d) dot = fmaf(qs[warp][d], to_f32<T>(kr[d]), dot);
            s = dot * p.scale;
        }
        const float mnew = fmaxf(m, warp_max(s));
        const float alpha = m == -INFINITY ? 0.f : expf(m - mnew);
        const float pt = t < L ? expf(s - mnew) : 0.f;
        l = l * alpha + pt;
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[i] *= alpha;
        m = mnew;
        const int nt = min(32, L - t0);
        for (int tt = 0; tt < nt; ++tt) {
            const float pp = __shfl_sync(0xffffffffu, pt, tt);
            const T* vr = gen_row<T>(p, vb, b, row, t0 + tt, g);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int d = lane + 32 * i;
                if (d < p.hd) acc[i] = fmaf(pp, to_f32<T>(vr[d]), acc[i]);
            }
        }
    }
    l = warp_sum(l);
    const float inv = L > 0 ? 1.f / l : 0.f;
    const int64_t ob = b * p.o_sb + j * p.o_sj + h * p.o_sh;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int d = lane + 32 * i;
        if (d < p.hd) store_from_f32(p.out, ob + d, p.out_dtype, acc[i] * inv);
    }
}

// ------------------------------------------------------------ host planning
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult qr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &qr) == cudaSuccess &&
            qr == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(ptr);
    });
    return fn;
}

int encode_kv_map(CUtensorMap* map, const void* base, int dtype, int64_t ntok, int hkv, int hd) {
    if (!base || (hd != 64 && hd != 128) || hkv < 1 || ntok < 1 || ntok > (int64_t(1) << 31) ||
        (dtype != SDL_BF16 && dtype != SDL_F16))
        return sdl::fail(SDL_ERR_UNSUPPORTED, "sdl_make_kv_tensor_map: needs bf16/f16, head_dim 64/128");
    if (reinterpret_cast<uintptr_t>(base) % 16 != 0)
        return sdl::fail(SDL_ERR_INVALID, "sdl_make_kv_tensor_map: base not 16-byte aligned");
    EncodeTiledFn fn = get_encode_fn();
    if (!fn) return sdl::fail(SDL_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
    cuuint64_t dims[4] = {64, (cuuint64_t)(hd / 64), (cuuint64_t)hkv, (cuuint64_t)ntok};
    cuuint64_t strides[3] = {128, (cuuint64_t)hd * 2, (cuuint64_t)hkv * hd * 2};
    cuuint32_t box[4] = {64, 1, 1, (cuuint32_t)kPage};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    CUresult r = fn(map, dtype == SDL_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4,
                    const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return sdl::fail(SDL_ERR_CUDA, "cuTensorMapEncodeTiled failed");
    return SDL_OK;
}

struct Plan {
    bool tc = false;
    int ntg = 1, wpg = 1, ncoltiles = 1, g_cta = 1, kvgroups = 1;
    int pps = 1, nsplit = 1;
    int stage_bytes = 0;
    size_t smem = 0;
    size_t ws_bytes = 0;
};

int sm_count() {
    static int n = 0;
    if (n == 0) {
        int dev = 0;
        if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) !=
                                                      cudaSuccess || n <= 0)
            n = 148;
    }
    return n;
}

bool tc_applicable(const sdl_attn_args* a) {
    if (a->force_generic) return false;
    if (a->dtype != SDL_BF16 && a->dtype != SDL_F16) return false;
    if (a->head_dim != 64 && a->head_dim != 128) return false;
    if (a->k_pool && a->block_size != kPage) return false;
    const int ratio = a->Hq / a->Hkv;
    // 32-bit q fragment loads need even strides.
    if ((a->q_sb | a->q_sj | a->q_sh) & 1) return false;
    if (reinterpret_cast<uintptr_t>(a->q) % 4) return false;
    (void)ratio;
    return true;
}

Plan make_plan(const sdl_attn_args* a) {
    Plan pl;
    pl.tc = tc_applicable(a);
    if (!pl.tc) return pl;
    const int ratio = a->Hq / a->Hkv;
    const int ncol = a->chunk * ratio;
    const int ntiles = (ncol + 7) / 8;
    // Eight query columns per consumer warp while the tiles fit the warp
    // budget: the 16-column variant needs ~165 registers, which caps a CTA
    // of it at one per SM; the 8-column variant runs three per SM.
    pl.ntg = ntiles > kMaxConsumerWarps ? 2 : 1;
    pl.wpg = std::min((ntiles + pl.ntg - 1) / pl.ntg, kMaxConsumerWarps);
    pl.ncoltiles = (ntiles + pl.wpg * pl.ntg - 1) / (pl.wpg * pl.ntg);
    const int DO = a->head_dim / 64;
    const int head_stage = 2 * DO * kBoxBytes;
    pl.g_cta = 1;
    for (int gc = a->Hkv; gc >= 1; --gc) {
        if (a->Hkv % gc) continue;
        if (gc * pl.wpg > kMaxConsumerWarps) continue;
        if ((size_t)kStages * gc * head_stage > 160 * 1024) continue;
        if (a->kv_heads_per_cta > 0 && gc > a->kv_heads_per_cta) continue;
        pl.g_cta = gc;
        break;
    }
    pl.kvgroups = a->Hkv / pl.g_cta;
    pl.stage_bytes = pl.g_cta * head_stage;
    pl.smem = (size_t)kStages * pl.stage_bytes + 1024 + 2 * kStages * sizeof(uint64_t);
    const int max_pages = std::max(1, (a->max_limit + kPage - 1) / kPage);
    const long base_ctas = (long)a->B * pl.ncoltiles * pl.kvgroups;
    const long target = (long)sm_count() * 4;
    int nsplit_target = (int)std::max(1L, (target + base_ctas - 1) / base_ctas);
    int pps = a->pages_per_split > 0 ? a->pages_per_split : std::max(4, (max_pages + nsplit_target - 1) / nsplit_target);
    for (;;) {
        pl.pps = pps;
        pl.nsplit = (max_pages + pps - 1) / pps;
        pl.ws_bytes = pl.nsplit > 1 ? (size_t)a->B * pl.nsplit * a->chunk * a->Hq * (a->head_dim + 2) * sizeof(float) : 0;
        if (a->pages_per_split > 0 || pl.ws_bytes <= a->workspace_bytes || pl.nsplit == 1 || !a->workspace) break;
        pps *= 2;
    }
    return pl;
}

template <int HD, int NTG, typename T>
int launch_tc_inst(const CUtensorMap& mk, const CUtensorMap& mv, const TcParams& tp, const Plan& pl, cudaStream_t st) {
    auto kern = attn_tc_kernel<HD, NTG, T>;
    static size_t configured = 0;
    if (pl.smem > configured) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pl.smem);
        // all of the unified L1/shared array as shared memory: the ring buffers,
        // not L1, decide how many CTAs an SM holds
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout,
                                     (int)cudaSharedmemCarveoutMaxShared);
        if (e != cudaSuccess) return sdl::fail(SDL_ERR_CUDA, cudaGetErrorString(e));
        configured = pl.smem;
    }
    dim3 grid(pl.nsplit, pl.ncoltiles * pl.kvgroups, tp.B);
    dim3 block((pl.g_cta * pl.wpg + 1) * 32);
    cudaError_t e = sdl::launch_pdl(kern, grid, block, pl.smem, st, mk, mv, tp);
    if (e != cudaSuccess) return sdl::fail(SDL_ERR_CUDA, cudaGetErrorString(e));
    return sdl::check_launch("attn_tc_kernel");
}

template <typename T>
int launch_tc_dtype(int hd, int ntg, const CUtensorMap& mk, const CUtensorMap& mv, const TcParams& tp, const Plan& pl,
                    cudaStream_t st) {
    if (hd == 64) return ntg == 2 ? launch_tc_inst<64, 2, T>(mk, mv, tp, pl, st) : launch_tc_inst<64, 1, T>(mk, mv, tp, pl, st);
    return ntg == 2 ? launch_tc_inst<128, 2, T>(mk, mv, tp, pl, st) : launch_tc_inst<128, 1, T>(mk, mv, tp, pl, st);
}

int validate(const sdl_attn_args* a) {
    if (!a || !a->q || !a->out || !a->starts || a->B < 0 || a->chunk < 1 || a->Hq < 1 || a->Hkv < 1 ||
        a->Hq % a->Hkv || a->head_dim < 1 || a->head_dim > 256)
        return sdl::fail(SDL_ERR_INVALID, "sdl_paged_attention: bad shape arguments");
    if (a->dtype != SDL_F32 && a->dtype != SDL_BF16 && a->dtype != SDL_F16)
        return sdl::fail(SDL_ERR_UNSUPPORTED, "sdl_paged_attention: unsupported dtype");
    if (a->out_dtype != SDL_F32 && a->out_dtype != SDL_BF16 && a->out_dtype != SDL_F16)
        return sdl::fail(SDL_ERR_UNSUPPORTED, "sdl_paged_attention: unsupported out dtype");
    if (a->k_pool) {
        if (!a->v_pool || !a->block_table || !a->rows || a->width < 1 || a->capacity < 1 || a->block_size < 1 ||
            a->layer < 0 || a->layer >= a->num_layers)
            return sdl::fail(SDL_ERR_INVALID, "sdl_paged_attention: bad paged-pool arguments");
        if ((int64_t)a->num_layers * a->capacity * a->block_size >= (int64_t(1) << 31))
            return sdl::fail(SDL_ERR_UNSUPPORTED, "sdl_paged_attention: pool exceeds 2^31 token rows");
    } else {
        if (!a->k_dense || !a->v_dense || a->kv_len < 1)
            return sdl::fail(SDL_ERR_INVALID, "sdl_paged_attention: bad dense K/V arguments");
    }
    return SDL_OK;
}

}  // namespace

extern "C" int sdl_make_kv_tensor_map(void* out_map128, const void* base, int32_t dtype, int64_t num_tokens_total,
                                      int32_t num_kv_heads, int32_t head_dim) {
    if (!out_map128) return sdl::fail(SDL_ERR_INVALID, "sdl_make_kv_tensor_map: out is NULL");
    CUtensorMap map;
    int rc = encode_kv_map(&map, base, dtype, num_tokens_total, num_kv_heads, head_dim);
    if (rc != SDL_OK) return rc;
    memcpy(out_map128, &map, sizeof(CUtensorMap));
    return SDL_OK;
}

extern "C" size_t sdl_attention_workspace_bytes(const sdl_attn_args* args) {
    if (validate(args) != SDL_OK) return 0;
    Plan pl = make_plan(args);
    if (!pl.tc) return 0;
    sdl_attn_args tmp = *args;
    tmp.workspace = nullptr;
    tmp.workspace_bytes = 0;
    return make_plan(&tmp).ws_bytes;
}

extern "C" int sdl_paged_attention(const sdl_attn_args* a, void* stream) {
    int rc = validate(a);
    if (rc != SDL_OK) return rc;
    if (a->B == 0) return SDL_OK;
    cudaStream_t st = sdl::as_stream(stream);
    const int ratio = a->Hq / a->Hkv;
    Plan pl = make_plan(a);
    if (pl.tc) {
        if (pl.nsplit > 1 && (!a->workspace || a->workspace_bytes < pl.ws_bytes))
            return sdl::fail(SDL_ERR_WORKSPACE, "sdl_paged_attention: workspace too small");
        CUtensorMap mk, mv;
        if (a->k_pool) {
            if (a->tmap_k && a->tmap_v) {
                memcpy(&mk, a->tmap_k, sizeof(CUtensorMap));
                memcpy(&mv, a->tmap_v, sizeof(CUtensorMap));
            } else {
                const int64_t ntok = (int64_t)a->num_layers * a->capacity * a->block_size;
                if ((rc = encode_kv_map(&mk, a->k_pool, a->dtype, ntok, a->Hkv, a->head_dim)) != SDL_OK) return rc;
                if ((rc = encode_kv_map(&mv, a->v_pool, a->dtype, ntok, a->Hkv, a->head_dim)) != SDL_OK) return rc;
            }
        } else {
            const int64_t ntok = (int64_t)a->B * a->kv_len;
            if ((rc = encode_kv_map(&mk, a->k_dense, a->dtype, ntok, a->Hkv, a->head_dim)) != SDL_OK) return rc;
            if ((rc = encode_kv_map(&mv, a->v_dense, a->dtype, ntok, a->Hkv, a->head_dim)) != SDL_OK) return rc;
        }
        TcParams tp;
        tp.q = a->q; tp.q_sb = a->q_sb; tp.q_sj = a->q_sj; tp.q_sh = a->q_sh;
        tp.out = a->out; tp.o_sb = a->o_sb; tp.o_sj = a->o_sj; tp.o_sh = a->o_sh; tp.out_dtype = a->out_dtype;
        tp.table = a->block_table; tp.width = a->width; tp.capacity = a->capacity; tp.layer = a->layer;
        tp.rows = a->rows; tp.starts = a->starts; tp.valid_rows = a->valid_rows;
        tp.dense = a->k_pool ? 0 : 1; tp.kv_len = a->kv_len;
        tp.B = a->B; tp.chunk = a->chunk; tp.Hq = a->Hq; tp.Hkv = a->Hkv; tp.ratio = ratio;
        tp.pps = pl.pps; tp.nsplit = pl.nsplit;
        tp.g_cta = pl.g_cta; tp.wpg = pl.wpg; tp.ncoltiles = pl.ncoltiles;
        tp.stage_bytes = pl.stage_bytes;
        tp.scale_log2 = a->scale * 1.4426950408889634f;
        tp.o_part = a->workspace;
        tp.ml_part = a->workspace ? a->workspace + (size_t)a->B * pl.nsplit * a->chunk * a->Hq * a->head_dim : nullptr;
        tp.err = a->err;
        if (a->dtype == SDL_BF16) rc = launch_tc_dtype<__nv_bfloat16>(a->head_dim, pl.ntg, mk, mv, tp, pl, st);
        else rc = launch_tc_dtype<__half>(a->head_dim, pl.ntg, mk, mv, tp, pl, st);
        if (rc != SDL_OK) return rc;
        if (pl.nsplit > 1) {
            const int rows = a->B * a->chunk * a->Hq;
            cudaError_t e = sdl::launch_pdl(attn_combine_kernel, dim3((rows + 3) / 4), dim3(128), 0, st, tp,
                                            (int)a->head_dim);
            if (e != cudaSuccess) return sdl::fail(SDL_ERR_CUDA, cudaGetErrorString(e));
            rc = sdl::check_launch("attn_combine_kernel");
        }
        return rc;
    }
    GenParams gp;
    gp.q = a->q; gp.q_sb = a->q_sb; gp.q_sj = a->q_sj; gp.q_sh = a->q_sh;
    gp.out = a->out; gp.o_sb = a->o_sb; gp.o_sj = a->o_sj; gp.o_sh = a->o_sh; gp.out_dtype = a->out_dtype;
    gp.k = a->k_pool ? a->k_pool : a->k_dense;
    gp.v = a->k_pool ? a->v_pool : a->v_dense;
    gp.table = a->block_table; gp.width = a->width; gp.capacity = a->capacity; gp.layer = a->layer;
    gp.bs = a->block_size;
    gp.rows = a->rows; gp.starts = a->starts; gp.valid_rows = a->valid_rows;
    gp.dense = a->k_pool ? 0 : 1; gp.kv_len = a->kv_len;
    gp.B = a->B; gp.chunk = a->chunk; gp.Hq = a->Hq; gp.Hkv = a->Hkv; gp.ratio = ratio; gp.hd = a->head_dim;
    gp.scale = a->scale; gp.err = a->err;
    dim3 grid((a->chunk * a->Hq + 3) / 4, a->B);
    if (a->dtype == SDL_F32) attn_generic_kernel<float><<<grid, 128, 0, st>>>(gp);
    else if (a->dtype == SDL_BF16) attn_generic_kernel<__nv_bfloat16><<<grid, 128, 0, st>>>(gp);
    else attn_generic_kernel<__half><<<grid, 128, 0, st>>>(gp);
    return sdl::check_launch("attn_generic_kernel");
}

// ------------------------------------------------- allocation-free variant
// Some callers cannot allocate device memory at call time: a serving runtime
// that hands all HBM to its own pool allocator at start-up (cudaMalloc then
// fails or fragments that pool), or a foreign-language host (FFI) that only
// owns the input and output buffers it passes in.  For them,
// sdl_paged_attention_noalloc keeps the split-K partials in this file-scope
// array instead of a caller workspace.  Every GPU that loads the library
// holds the array (kNoAllocScratchBytes) until the process exits.
constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;  // 8 MiB
static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchBytes / sizeof(float)];

namespace {
std::mutex g_noalloc_mu;
float* g_noalloc_ptr[128] = {nullptr};

// Device address of g_noalloc_scratch on the current device.  The host-side
// symbol is only a stand-in, so the address is looked up once per device
// (with that device current) and cached.
int noalloc_scratch(float** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return sdl::fail(SDL_ERR_CUDA, cudaGetErrorString(e));
    if (dev < 0 || dev >= 128) return sdl::fail(SDL_ERR_INVALID, "sdl_paged_attention_noalloc: device ordinal >= 128");
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (g_noalloc_ptr[dev] == nullptr) {
        void* ptr = nullptr;
        e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
        if (e != cudaSuccess || ptr == nullptr)
            return sdl::fail(SDL_ERR_CUDA, "cudaGetSymbolAddress(g_noalloc_scratch) failed");
        g_noalloc_ptr[dev] = static_cast<float*>(ptr);
    }
    *out = g_noalloc_ptr[dev];
    return SDL_OK;
}
}  // namespace

extern "C" size_t sdl_noalloc_scratch_bytes(void) { return kNoAllocScratchBytes; }

extern "C" int sdl_paged_attention_noalloc(const sdl_attn_args* args, void* stream) {
    int rc = validate(args);
    if (rc != SDL_OK) return rc;
    sdl_attn_args a = *args;
    a.workspace = nullptr;
    a.workspace_bytes = 0;
    const size_t need = sdl_attention_workspace_bytes(&a);
    if (need > kNoAllocScratchBytes) {
        char msg[256];
        snprintf(msg, sizeof(msg),
                 "sdl_paged_attention_noalloc: this call needs %zu bytes of split-K scratch, more than the "
                 "%zu-byte static scratch; pass a workspace to sdl_paged_attention instead",
                 need, kNoAllocScratchBytes);
        return sdl::fail(SDL_ERR_WORKSPACE, msg);
    }
    if (need > 0) {
        float* scratch = nullptr;
        if ((rc = noalloc_scratch(&scratch)) != SDL_OK) return rc;
        a.workspace = scratch;
        a.workspace_bytes = kNoAllocScratchBytes;
    }
    return sdl_paged_attention(&a, stream);
}

extern "C" int sdl_paged_decode(const sdl_attn_args* args, void* stream) {
    if (args && args->chunk != 1) return sdl::fail(SDL_ERR_INVALID, "sdl_paged_decode: chunk must be 1");
    return sdl_paged_attention(args, stream);
}

extern "C" int sdl_paged_verify(const sdl_attn_args* args, void* stream) { return sdl_paged_attention(args, stream); }

extern "C" int sdl_prefill_chunk(const sdl_attn_args* args, void* stream) { return sdl_paged_attention(args, stream); }
