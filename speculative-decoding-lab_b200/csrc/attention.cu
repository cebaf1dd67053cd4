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
//    in the log2 domain with warp-shuffle column reductions and a lazy
//    running max; P is carried as a hi+lo pair of 16-bit values for fp32
//    output (the PV product keeps ~16 mantissa bits) and rounded once for
//    16-bit output.  Splits write fp32 partials; attn_combine_kernel merges
//    them.
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
#include <type_traits>
#include <utility>
#include <vector>

namespace {

constexpr int kPage = 16;          // tokens per TMA page (= block_size on the TC path)
constexpr int kStages = 4;         // TMA ring depth
constexpr int kMaxConsumerWarps = 8;
constexpr int kBoxBytes = kPage * 128;  // one [16 tokens][64 cols] 16-bit box
constexpr uint32_t kWaitLimit = 1u << 20;
constexpr int kMaxClusterSplits = 16;  // splits of one row merged on chip (non-portable cluster size)
constexpr float kLazyLog2 = 8.f;   // running-max slack of the mma.sync kernel's softmax (log2 units)
constexpr int kCombineOneRound = 16;  // split merge: splits whose partials one round of loads covers

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
    int ring_bytes;  // shared bytes before the mbarriers: the TMA ring, reused for cluster partials
    int stages;      // ring depth of the rows-on-M kernel
    int cluster;     // 1: the splits of a row form one cluster and merge their partials on chip
    float scale_log2;
    float* o_part;
    float* ml_part;
    int4* sk_table;  // persistent tcgen05 kernel: per (sequence, kv head) {first tile, tiles, slot, slots}
    // fused K/V append (mma.sync kernel): new rows [B*chunk][Hkv][d] written at
    // positions starts[b] + j before they are attended; NULL = no append
    char* k_pool;
    char* v_pool;
    const char* k_new;
    const char* v_new;
    int64_t new_stride;  // bytes between consecutive new rows
    const char* k_src;   // K and V rows attended (the pool, or the dense tensors): register-direct kernel
    const char* v_src;
    int32_t* err;
    // RoPE inside the launch (mma.sync kernels with the fused append): cos /
    // sin row b*chunk + j (rope_stride elements apart) rotates q as it is
    // loaded and k_new as it is stored; NULL = q and k_new are used as given
    const char* rope_cos;
    const char* rope_sin;
    int64_t rope_stride;
    int overlap;  // distinct layers back to back: dependents start early, older pages stream before the wait
};

SDL_DEV uint32_t ld_u32(const void* p) { return *reinterpret_cast<const uint32_t*>(p); }

// Rotate-half RoPE of one element, the framework chain's roundings
// (x * cos + rotate_half(x) * sin with each product rounded to T; the caller
// rounds the sum): x is this dim's value, y its partner's (dim +- d/2), and
// rotate_half(x) here is -y in the first half of the head, y in the second.
template <typename T>
SDL_DEV float rope_elem(float x, float y, float c, float s, bool first_half) {
    const float a = round_trip<T>(__fmul_rn(x, c));
    const float b = round_trip<T>(__fmul_rn(first_half ? -y : y, s));
    return __fadd_rn(a, b);
}

template <typename T> SDL_DEV float half_lo(uint32_t v) { return to_f32<T>(reinterpret_cast<const T*>(&v)[0]); }
template <typename T> SDL_DEV float half_hi(uint32_t v) { return to_f32<T>(reinterpret_cast<const T*>(&v)[1]); }

// Two dims of a row held as packed pairs: x1 = dims (e, e+1) of the first
// half, x2 = dims (e+half, e+half+1); cr / sr the row's cos / sin.
template <typename T>
SDL_DEV void rope_u32(uint32_t& x1, uint32_t& x2, const T* cr, const T* sr, int e, int half) {
    const uint32_t c1 = ld_u32(cr + e), s1 = ld_u32(sr + e), c2 = ld_u32(cr + e + half), s2 = ld_u32(sr + e + half);
    const float a0 = half_lo<T>(x1), a1 = half_hi<T>(x1), b0 = half_lo<T>(x2), b1 = half_hi<T>(x2);
    x1 = pack2<T>(rope_elem<T>(a0, b0, half_lo<T>(c1), half_lo<T>(s1), true),
                  rope_elem<T>(a1, b1, half_hi<T>(c1), half_hi<T>(s1), true));
    x2 = pack2<T>(rope_elem<T>(b0, a0, half_lo<T>(c2), half_lo<T>(s2), false),
                  rope_elem<T>(b1, a1, half_hi<T>(c2), half_hi<T>(s2), false));
}

// Eight dims of a row as a 16-byte piece: own, the partner piece (dims +- d/2)
// and the piece's cos / sin.
template <typename T>
SDL_DEV uint4 rope_piece(uint4 own, uint4 partner, uint4 c, uint4 sn, bool first_half) {
    const uint32_t* o = reinterpret_cast<const uint32_t*>(&own);
    const uint32_t* q = reinterpret_cast<const uint32_t*>(&partner);
    const uint32_t* cc = reinterpret_cast<const uint32_t*>(&c);
    const uint32_t* ss = reinterpret_cast<const uint32_t*>(&sn);
    uint4 r;
    uint32_t* rr = reinterpret_cast<uint32_t*>(&r);
#pragma unroll
    for (int w = 0; w < 4; ++w)
        rr[w] = pack2<T>(rope_elem<T>(half_lo<T>(o[w]), half_lo<T>(q[w]), half_lo<T>(cc[w]), half_lo<T>(ss[w]),
                                      first_half),
                         rope_elem<T>(half_hi<T>(o[w]), half_hi<T>(q[w]), half_hi<T>(cc[w]), half_hi<T>(ss[w]),
                                      first_half));
    return r;
}

// Fused append: copies the K and V rows of one kv head for up to kAppendBatch
// new positions (byte offsets `src` into k_new / v_new and `dst` into the
// pools; dst < 0 skips a position; `nrow` the new-row index b*chunk + j).
// Lanes own 16-byte pieces (K pieces, then V pieces) and issue every load of
// the batch before any store, so a batch costs one memory round trip.  With
// RoPE a K lane also loads its rotate-half partner piece (dims +- d/2; the
// piece count is a power of two) and its cos / sin pieces.
constexpr int kAppendBatch = 4;
template <int HD, typename T>
SDL_DEV void copy_new_rows(const TcParams& p, int lane, const int64_t (&src)[kAppendBatch],
                           const int64_t (&dst)[kAppendBatch], const int (&nrow)[kAppendBatch], int n) {
    constexpr int kChunks = HD * (int)sizeof(T) / 16;
    if (lane >= 2 * kChunks) return;
    const bool isv = lane >= kChunks;
    const int c = lane % kChunks;
    const int cb = c * 16;
    const char* s0 = isv ? p.v_new : p.k_new;
    char* d0 = isv ? p.v_pool : p.k_pool;
    if (!isv && p.rope_cos != nullptr) {
        // one row at a time: four 16-byte loads per row, few registers (the
        // batch arrays would be live across the whole producer)
        const int pcb = (c ^ (kChunks / 2)) * 16;
#pragma unroll 1
        for (int u = 0; u < n; ++u) {
            if (dst[u] < 0) continue;
            const int64_t ro = (int64_t)nrow[u] * p.rope_stride * (int64_t)sizeof(T) + cb;
            const uint4 own = *reinterpret_cast<const uint4*>(s0 + src[u] + cb);
            const uint4 par = *reinterpret_cast<const uint4*>(s0 + src[u] + pcb);
            const uint4 cv = *reinterpret_cast<const uint4*>(p.rope_cos + ro);
            const uint4 sv = *reinterpret_cast<const uint4*>(p.rope_sin + ro);
            *reinterpret_cast<uint4*>(d0 + dst[u] + cb) = rope_piece<T>(own, par, cv, sv, c < kChunks / 2);
        }
        return;
    }
    uint4 v[kAppendBatch];
#pragma unroll
    for (int u = 0; u < kAppendBatch; ++u)
        if (u < n && dst[u] >= 0) v[u] = *reinterpret_cast<const uint4*>(s0 + src[u] + cb);
#pragma unroll
    for (int u = 0; u < kAppendBatch; ++u)
        if (u < n && dst[u] >= 0) *reinterpret_cast<uint4*>(d0 + dst[u] + cb) = v[u];
}

// 8-column warps: at least two 288-thread CTAs per SM (<= 112 registers), so
// the 192-thread verify CTAs stay at three per SM.
template <int HD, int NTG, typename T>
__global__ void __launch_bounds__((kMaxConsumerWarps + 1) * 32, NTG == 1 ? 2 : 1)
attn_tc_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv, const TcParams p) {
    constexpr int DO = HD / 64;
    constexpr int KSTEPS = HD / 16;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + p.ring_bytes);
    uint64_t* empty = full + kStages;
    uint64_t* xbar = empty + kStages;  // cluster merge: [0] partials stored, [1] partials read
    __shared__ int s_abort_flag;
    volatile int* s_abort = &s_abort_flag;

    if (p.overlap) pdl_launch_dependents();  // the next layer's launch may become resident now
    const int b = blockIdx.z;
    const int split = blockIdx.x;
    const int coltile = blockIdx.y % p.ncoltiles;
    const int kvgrp = blockIdx.y / p.ncoltiles;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ncons = p.g_cta * p.wpg;

    // Launched as a programmatic dependent, so this CTA may start while the
    // preceding kernel runs.  The row metadata (starts, valid_rows, rows) and
    // the block table are read before griddepcontrol.wait: no kernel of this
    // library that lets its dependents start early (attention, split merge,
    // K/V append, sampler) writes them, and the kernels that do (reserve,
    // release, commit) run to completion before a dependent starts.  Q, the
    // new K/V rows and the pool pages are read only after the wait.
    const int start = p.starts[b];
    const int nvalid = p.valid_rows ? min(p.valid_rows[b], p.chunk) : p.chunk;
    const int ncol = p.chunk * p.ratio;
    const int tile_cols = p.wpg * NTG * 8;
    const int col0 = coltile * tile_cols;
    int lmax = 0;
    if (col0 < ncol && col0 / p.ratio < nvalid) {
        const int col_last = min(col0 + tile_cols, ncol) - 1;
        const int j_last = min(col_last / p.ratio, nvalid - 1);
        lmax = start + j_last + 1;
    }
    const int npages = lmax > 0 ? (lmax + kPage - 1) / kPage : 0;
    const int pbeg = split * p.pps;
    const int pend = min(npages, pbeg + p.pps);
    // splits holding pages of this (sequence, kv-head group, column tile):
    // ranks 0..nact-1.  A span past the grid (max_limit below some
    // starts[b] + chunk) is reported and its excess pages are not attended.
    int nact = (npages + p.pps - 1) / p.pps;
    if (nact > p.nsplit) {
        if (threadIdx.x == 0 && split == 0) sdl_raise(p.err, SDL_DEVERR_BAD_INDEX);
        nact = p.nsplit;
    }
    if (p.cluster) {
        // The cluster is the row's splits.  Barriers for the on-chip merge are
        // initialised before any CTA of the cluster may signal them, and every
        // thread of every CTA passes this point before any CTA leaves.
        if (threadIdx.x == 0 && pbeg < pend && nact > 1) {
            mbar_init(&xbar[0], nact - 1);
            mbar_init(&xbar[1], nact - 1);
            fence_mbar_init();
        }
        cluster_sync_all();
    }
    if (lmax <= 0 || pbeg >= pend) return;
    const int np = pend - pbeg;
    const int row = p.dense ? 0 : p.rows[b];
    // Pool token row of page pbeg + i (producer lanes; out-of-range entries raise and read row 0).
    auto page_tok = [&](int i) -> int {
        const int pg = pbeg + i;
        if (p.dense) return b * p.kv_len + pg * kPage;
        int phys = pg < p.width ? p.table[(int64_t)row * p.width + pg] : -1;
        if (phys < 0 || phys >= p.capacity) { sdl_raise(p.err, SDL_DEVERR_BAD_INDEX); phys = 0; }
        return (p.layer * p.capacity + phys) * kPage;
    };
    const int tok_first = (warp == ncons && lane < np) ? page_tok(lane) : 0;  // the first 32 pages

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
        // Fused append: every new row whose page lies in this CTA's range is
        // written for this CTA's kv heads (CTAs sharing a page write the same
        // bytes) and made visible to this CTA's own TMA reads, just before the
        // first page that holds one is issued -- the earlier pages' copies are
        // in flight meanwhile.
        const int app_page = p.k_new != nullptr ? max(pbeg, start / kPage) : pend;
        // Layers back to back (p.overlap) with the fused append: the pages
        // before the first new row hold keys of earlier, completed launches
        // (the caller's contract), so the first ring stages of them are
        // issued before griddepcontrol.wait and stream while the preceding
        // kernel drains.  Without k_new a separate append may just have
        // written any page.
        const int npre = p.overlap && p.k_new != nullptr ? min(kStages, min(np, app_page - pbeg)) : 0;
        for (int i = 0; i < npre; ++i) {
            const int t0 = __shfl_sync(0xffffffffu, tok_first, i);
            if (lane == 0) {
                mbar_arrive_expect_tx(&full[i], p.stage_bytes);
                uint8_t* sbuf = smem + i * p.stage_bytes;
                for (int gi = 0; gi < p.g_cta; ++gi) {
                    const int g = kvgrp * p.g_cta + gi;
                    uint8_t* kb = sbuf + gi * (2 * DO * kBoxBytes);
#pragma unroll
                    for (int dd = 0; dd < DO; ++dd) {
                        tma_load_4d(kb + dd * kBoxBytes, &tmk, &full[i], 0, dd, g, t0);
                        tma_load_4d(kb + (DO + dd) * kBoxBytes, &tmv, &full[i], 0, dd, g, t0);
                    }
                }
            }
            __syncwarp();
        }
        pdl_wait();
        auto append_rows = [&]() {
            const int row_bytes = p.Hkv * HD * (int)sizeof(T);
            for (int j0 = 0; j0 < nvalid; j0 += kAppendBatch) {
                // lane u < kAppendBatch resolves position start + j0 + u: its pool token row, or -1
                int64_t trow = -1;
                if (lane < kAppendBatch && j0 + lane < nvalid) {
                    const int pos = start + j0 + lane, pg = pos / kPage;
                    if (pg >= pbeg && pg < pend) {
                        const int phys = pg < p.width ? p.table[(int64_t)row * p.width + pg] : -1;
                        if (phys < 0 || phys >= p.capacity) sdl_raise(p.err, SDL_DEVERR_BAD_INDEX);
                        else trow = (int64_t)(p.layer * p.capacity + phys) * kPage + pos % kPage;
                    }
                }
                int64_t tr[kAppendBatch];
#pragma unroll
                for (int u = 0; u < kAppendBatch; ++u) tr[u] = __shfl_sync(0xffffffffu, trow, u);
                for (int gi = 0; gi < p.g_cta; ++gi) {
                    const int hoff = (kvgrp * p.g_cta + gi) * HD * (int)sizeof(T);
                    int64_t src[kAppendBatch], dst[kAppendBatch];
                    int nrow[kAppendBatch];
#pragma unroll
                    for (int u = 0; u < kAppendBatch; ++u) {
                        nrow[u] = b * p.chunk + j0 + u;
                        src[u] = (int64_t)nrow[u] * p.new_stride + hoff;
                        dst[u] = tr[u] >= 0 ? tr[u] * row_bytes + hoff : -1;
                    }
                    copy_new_rows<HD, T>(p, lane, src, dst, nrow, min(kAppendBatch, nvalid - j0));
                }
            }
            asm volatile("fence.proxy.async.global;" ::: "memory");
            __syncwarp();
        };
        int issued = 0;
        bool stop = false;
        for (int i0 = 0; i0 < np && !stop; i0 += 32) {
            const int tok0 = i0 == 0 ? tok_first : (i0 + lane < np ? page_tok(i0 + lane) : 0);
            const int cnt = min(32, np - i0);
            for (int k = 0; k < cnt; ++k) {
                const int t0 = __shfl_sync(0xffffffffu, tok0, k);
                const int i = i0 + k;
                const int st = i % kStages;
                if (i < npre) { issued = i + 1; continue; }  // issued before the wait
                if (pbeg + i == app_page) append_rows();
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
    pdl_wait();  // Q comes from the preceding kernels
    const int gi = warp / p.wpg, wc = warp % p.wpg;
    const int g = kvgrp * p.g_cta + gi;
    const int cbase = col0 + wc * NTG * 8;
    const int tq = lane & 3, grp = lane >> 2;

    uint32_t qf[KSTEPS][NTG][2];
#pragma unroll
    for (int nt = 0; nt < NTG; ++nt) {
        const int col = cbase + nt * 8 + grp;
        const bool ok = col < ncol && col / p.ratio < nvalid;
        const int j = ok ? col / p.ratio : 0;
        const T* qp = nullptr;
        if (ok) qp = reinterpret_cast<const T*>(p.q) + b * p.q_sb + j * p.q_sj + (g * p.ratio + col % p.ratio) * p.q_sh;
#pragma unroll
        for (int ks = 0; ks < KSTEPS; ++ks) {
            qf[ks][nt][0] = ok ? ld_u32(qp + ks * 16 + 2 * tq) : 0u;
            qf[ks][nt][1] = ok ? ld_u32(qp + ks * 16 + 8 + 2 * tq) : 0u;
        }
        if (ok && p.rope_cos != nullptr) {  // dims e and e + d/2 sit in k-steps ks and ks + KSTEPS/2
            const int64_t ro = (int64_t)(b * p.chunk + j) * p.rope_stride;
            const T* cr = reinterpret_cast<const T*>(p.rope_cos) + ro;
            const T* sr = reinterpret_cast<const T*>(p.rope_sin) + ro;
#pragma unroll
            for (int ks = 0; ks < KSTEPS / 2; ++ks) {
                rope_u32<T>(qf[ks][nt][0], qf[ks + KSTEPS / 2][nt][0], cr, sr, ks * 16 + 2 * tq, HD / 2);
                rope_u32<T>(qf[ks][nt][1], qf[ks + KSTEPS / 2][nt][1], cr, sr, ks * 16 + 8 + 2 * tq, HD / 2);
            }
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
    int lim_min = lmax;  // smallest key limit among this warp's valid columns
#pragma unroll
    for (int nt = 0; nt < NTG; ++nt) lim_min = min(lim_min, min(lim[nt][0], lim[nt][1]));
    lim_min = __reduce_min_sync(0xffffffffu, lim_min);
    float acc[KSTEPS][NTG][4];
#pragma unroll
    for (int mt = 0; mt < KSTEPS; ++mt)
#pragma unroll
        for (int nt = 0; nt < NTG; ++nt)
#pragma unroll
            for (int r = 0; r < 4; ++r) acc[mt][nt][r] = 0.f;

    const uint32_t sbase = smem_u32(smem);
    const int mi = lane >> 3, mr = lane & 7;
    // This lane's ldmatrix row offsets within a 2 KB swizzled box: key row t,
    // 16-byte chunk (2q + h) XOR (t & 7) for the four 16-column steps q of a
    // 64-column half (K: rows t = mr + 8 (mi & 1), h = mi >> 1; V transposed:
    // t = mr + 8 (mi >> 1), h = mi & 1).
    uint32_t koff[4], voff[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const int tk = mr + ((mi & 1) << 3), tv = mr + ((mi >> 1) << 3);
        koff[q] = tk * 128 + (((2 * q + (mi >> 1)) ^ (tk & 7)) << 4);
        voff[q] = tv * 128 + (((2 * q + (mi & 1)) ^ (tv & 7)) << 4);
    }
    // P as a hi + lo pair for fp32 output (~16 mantissa bits of every weight);
    // once rounded for 16-bit outputs, whose own rounding bounds the result.
    const bool p_split = p.out_dtype == SDL_F32;
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
            uint32_t a[4];
            ldmatrix_x4(kbase + koff[ks & 3] + (ks >> 2) * kBoxBytes, a[0], a[1], a[2], a[3]);
#pragma unroll
            for (int nt = 0; nt < NTG; ++nt) mma_16816<T>(s[nt], a, qf[ks][nt][0], qf[ks][nt][1]);
        }

        // Online softmax per query column (log2 domain) with a lazy running
        // max: m_run only moves -- and O, l are rescaled -- when a page's max
        // exceeds it by more than 2^kLazyLog2, so p <= 2^kLazyLog2 and most
        // pages skip the rescale.  Pages wholly below every column's key
        // limit skip the causal mask.
        const int pos_lo = (pbeg + i) * kPage + grp, pos_hi = pos_lo + 8;
        const bool whole = (pbeg + i + 1) * kPage <= lim_min;
        float mx[NTG][2];
        bool need = false;
#pragma unroll
        for (int nt = 0; nt < NTG; ++nt)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                if (!whole) {
                    if (pos_lo >= lim[nt][e]) s[nt][e] = -INFINITY;
                    if (pos_hi >= lim[nt][e]) s[nt][2 + e] = -INFINITY;
                }
                float m = fmaxf(s[nt][e], s[nt][2 + e]);
                m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 4));
                m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 8));
                m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 16));
                mx[nt][e] = m * p.scale_log2;
                need |= mx[nt][e] > m_run[nt][e] + kLazyLog2;
            }
        if (__any_sync(0xffffffffu, need)) {
#pragma unroll
            for (int nt = 0; nt < NTG; ++nt)
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    if (!(mx[nt][e] > m_run[nt][e] + kLazyLog2)) continue;
                    const float alpha = ex2_approx(m_run[nt][e] - mx[nt][e]);  // 0 on the first page
                    m_run[nt][e] = mx[nt][e];
                    l_run[nt][e] *= alpha;
#pragma unroll
                    for (int mt = 0; mt < KSTEPS; ++mt) {
                        acc[mt][nt][e] *= alpha;
                        acc[mt][nt][2 + e] *= alpha;
                    }
                }
        }
        uint32_t pb[NTG][2], pl[NTG][2];
#pragma unroll
        for (int nt = 0; nt < NTG; ++nt) {
            float pv[4];
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                // a column that has seen only masked keys keeps m_run = -inf; its p is 0
                const float muse = m_run[nt][e] == -INFINITY ? 0.f : m_run[nt][e];
                pv[e] = ex2_approx(fmaf(s[nt][e], p.scale_log2, -muse));
                pv[2 + e] = ex2_approx(fmaf(s[nt][2 + e], p.scale_log2, -muse));
                l_run[nt][e] += pv[e] + pv[2 + e];
            }
            pb[nt][0] = movmatrix_trans(pack2<T>(pv[0], pv[1]));
            pb[nt][1] = movmatrix_trans(pack2<T>(pv[2], pv[3]));
            if (p_split) {
                const float h0 = round_trip<T>(pv[0]), h1 = round_trip<T>(pv[1]);
                const float h2 = round_trip<T>(pv[2]), h3 = round_trip<T>(pv[3]);
                pl[nt][0] = movmatrix_trans(pack2<T>(pv[0] - h0, pv[1] - h1));
                pl[nt][1] = movmatrix_trans(pack2<T>(pv[2] - h2, pv[3] - h3));
            }
        }

        // O^T[d][col] += sum_t V[t][d] P^T[t][col]
#pragma unroll
        for (int mt = 0; mt < KSTEPS; ++mt) {
            uint32_t a[4];
            ldmatrix_x4_trans(vbase + voff[mt & 3] + (mt >> 2) * kBoxBytes, a[0], a[1], a[2], a[3]);
#pragma unroll
            for (int nt = 0; nt < NTG; ++nt) {
                mma_16816<T>(acc[mt][nt], a, pb[nt][0], pb[nt][1]);
                if (p_split) mma_16816<T>(acc[mt][nt], a, pl[nt][0], pl[nt][1]);
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[st]);
    }
    __syncthreads();
    pdl_launch_dependents();  // the split merge may be scheduled during the epilogue
    const bool cmerge = p.cluster && nact > 1;
    if ((aborted || *s_abort) && !cmerge) return;
    const bool failed = aborted || *s_abort;

    // Cluster merge: partials go to this CTA's shared memory (the ring is
    // free now), row stride PST floats, then m and l per local column.
    constexpr int PST = HD + 4;
    const int ncl = ncons * NTG * 8;
    float* part = reinterpret_cast<float*>(smem);
    float* part_m = part + ncl * PST;
    float* part_l = part_m + ncl;

    // Epilogue: finished rows write the output, split rows write partials.
    if (!failed) {
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
            } else if (cmerge) {
                const int lc = gi * tile_cols + (col - col0);
                float* op = part + lc * PST;
#pragma unroll
                for (int mt = 0; mt < KSTEPS; ++mt) {
                    op[mt * 16 + grp] = acc[mt][nt][e];
                    op[mt * 16 + grp + 8] = acc[mt][nt][2 + e];
                }
                if (grp == 0) {
                    part_m[lc] = m_run[nt][e];
                    part_l[lc] = l;
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
    if (!cmerge) return;

    // On-chip merge.  Every active split signals the others once its partials
    // are stored; split r then merges the local columns lc = r (mod nact)
    // from all splits' shared memory, and no CTA leaves before every split
    // has finished reading it.  All waits are bounded.
    fence_acq_rel_cluster();
    named_bar_sync(1, ncons * 32);
    const uint32_t rank = cluster_ctarank();
    if (threadIdx.x == 0) {
        for (int r = 0; r < nact; ++r)
            if (r != (int)rank) mbar_arrive_remote(mapa_shared(smem_u32(&xbar[0]), r));
    }
    bool ready = mbar_wait_cluster_bounded(&xbar[0], 0, kWaitLimit);
    if (!ready && lane == 0) sdl_raise(p.err, SDL_DEVERR_TIMEOUT);
    if (ready && !failed) {
        constexpr int DPL = HD / 32;  // head dims per lane
        for (int lc = (int)rank + warp * nact; lc < ncl; lc += ncons * nact) {
            const int gi_c = lc / tile_cols;
            const int col = col0 + lc % tile_cols;
            if (col >= ncol) continue;
            const int j = col / p.ratio;
            if (j >= nvalid) continue;
            const int L = start + j + 1;
            const int ns_c = min(nact, ((L + kPage - 1) / kPage + p.pps - 1) / p.pps);
            if (ns_c <= 1) continue;
            const uint32_t a_m = smem_u32(part_m + lc), a_l = smem_u32(part_l + lc);
            const uint32_t a_o = smem_u32(part + lc * PST + lane * DPL);
            float M = -INFINITY;
            for (int r = 0; r < ns_c; ++r) M = fmaxf(M, ld_cluster_f32(mapa_shared(a_m, r)));
            float den = 0.f, o[DPL];
#pragma unroll
            for (int k = 0; k < DPL; ++k) o[k] = 0.f;
#pragma unroll 4
            for (int r = 0; r < ns_c; ++r) {
                const float mr_ = ld_cluster_f32(mapa_shared(a_m, r));
                const float w = mr_ == -INFINITY ? 0.f : ex2_approx(mr_ - M);
                den = fmaf(w, ld_cluster_f32(mapa_shared(a_l, r)), den);
                if constexpr (DPL == 4) {
                    const float4 v = ld_cluster_f32x4(mapa_shared(a_o, r));
                    o[0] = fmaf(w, v.x, o[0]); o[1] = fmaf(w, v.y, o[1]);
                    o[2] = fmaf(w, v.z, o[2]); o[3] = fmaf(w, v.w, o[3]);
                } else {
                    const float2 v = ld_cluster_f32x2(mapa_shared(a_o, r));
                    o[0] = fmaf(w, v.x, o[0]); o[1] = fmaf(w, v.y, o[1]);
                }
            }
            const float inv = 1.f / den;
            const int h = (kvgrp * p.g_cta + gi_c) * p.ratio + col % p.ratio;
            const int64_t ob = b * p.o_sb + j * p.o_sj + h * p.o_sh + lane * DPL;
#pragma unroll
            for (int k = 0; k < DPL; ++k) store_from_f32(p.out, ob + k, p.out_dtype, o[k] * inv);
        }
    }
    named_bar_sync(1, ncons * 32);  // this CTA's reads of the other splits are done
    if (threadIdx.x == 0) {
        for (int r = 0; r < nact; ++r)
            if (r != (int)rank) mbar_arrive_remote(mapa_shared(smem_u32(&xbar[1]), r));
        if (!mbar_wait_cluster_bounded(&xbar[1], 0, kWaitLimit)) sdl_raise(p.err, SDL_DEVERR_TIMEOUT);
    }
}

// ---------------------------------------------------------------------------
// Register-direct decode kernel: keys on the MMA M dimension like
// attn_tc_kernel, but each thread loads its mma.sync fragment elements
// straight from the pool rows as 16-byte pieces -- no TMA, no shared-memory
// ring, no barrier inside the page loop.  One CTA per (split, group of
// g_cta kv heads, sequence) for blocks of at most kDirCols query columns per
// kv head; warp w attends kv head w % g_cta, the kDirWarps / g_cta warps of
// a head take the split's pages round-robin, each with its own online
// softmax, and merge through shared memory at the end.  With g_cta = Hkv
// the heads' halves of a token row are read together by sibling warps.
//
// Fragment layout (m16n8k16, g = lane / 4, c = lane % 4):
//  * S^T = K Q^T.  The head dimension is summed over, so it is permuted the
//    same way in K (A) and Q (B): k-step 2j + h takes, for this thread, dims
//    32j + 8c + 4h + {0,1} (fragment columns 2c, 2c+1) and + {2,3} (columns
//    2c+8, 2c+9).  One 16-byte piece of a K row (dims 32j + 8c .. +8) then
//    feeds two k-steps, and a quad of lanes reads 64 contiguous bytes.
//  * O^T += V^T P^T.  The M rows of O^T are head dims, permuted so that M
//    tile 4u + w, rows g and g + 8, are dims 64u + 8g + 2w and + 1: word w of
//    the 16-byte piece (dims 64u + 8g .. +8) of a V row holds both.  The A
//    fragment pairs two keys per register, so the words of keys 2c, 2c+1
//    (and 2c+8, 2c+9) are interleaved with byte permutes.
// The next page's K (after this page's S) and V (after this page's P V) are
// loaded while the current page is computed.
constexpr int kDirWarps = 4;
constexpr int kDirCols = 8;  // query columns (chunk * ratio) one CTA covers

template <int I> SDL_DEV uint32_t u4_word(const uint4& v) {
    if constexpr (I == 0) return v.x;
    else if constexpr (I == 1) return v.y;
    else if constexpr (I == 2) return v.z;
    else return v.w;
}

// Three CTAs per SM at head_dim 128 (the two pages in flight need ~140
// registers), four at 64.
template <int HD, typename T>
__global__ void __launch_bounds__(kDirWarps * 32, HD == 128 ? 3 : 4)
attn_direct_kernel(const TcParams p) {
    constexpr int KC = HD / 32;              // 16-byte K pieces per key row and thread
    constexpr int VC = HD / 64;              // 16-byte V pieces per key and thread
    constexpr int MT = HD / 16;              // k-steps of S^T = M tiles of O^T
    constexpr int RB = HD * (int)sizeof(T);  // bytes of one kv head's row
    __shared__ __align__(16) float s_part[kDirWarps][kDirCols][HD + 4];
    __shared__ float s_m[kDirWarps][kDirCols], s_l[kDirWarps][kDirCols];

    const int split = blockIdx.x, b = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tq = lane & 3, grp = lane >> 2;
    const int G = p.g_cta, WH = kDirWarps / G;  // kv heads per CTA, warps per head
    const int gi = warp % G, wi = warp / G;
    const int g = blockIdx.y * G + gi;

    // Row metadata and the block table are read before griddepcontrol.wait
    // (as in attn_tc_kernel: no early-starting kernel of this library writes
    // them); Q, the new rows and the pool pages after it.
    const int start = p.starts[b];
    const int nvalid = p.valid_rows ? min(p.valid_rows[b], p.chunk) : p.chunk;
    const int ncol = p.chunk * p.ratio;
    const int lmax = nvalid > 0 ? start + nvalid : 0;
    if (lmax <= 0) return;
    const int npages = (lmax + kPage - 1) / kPage;
    if (split == 0 && threadIdx.x == 0 && (npages + p.pps - 1) / p.pps > p.nsplit)
        sdl_raise(p.err, SDL_DEVERR_BAD_INDEX);  // span past the grid: the excess pages are not attended
    const int pbeg = split * p.pps;
    const int pend = min(npages, pbeg + p.pps);
    if (pbeg >= pend) return;
    const int np = pend - pbeg;
    const int my_n = wi < np ? (np - wi + WH - 1) / WH : 0;
    const int row = p.dense ? 0 : p.rows[b];
    const int klim = p.dense ? min(lmax, p.kv_len) : lmax;  // keys loaded (the rest read as zero)
    const int64_t rs = (int64_t)p.Hkv * RB;                  // bytes of one token row
    // Pool token row of this warp's k-th page (out-of-range entries raise and read row 0).
    auto page_tok = [&](int k) -> int {
        const int pg = pbeg + wi + k * WH;
        if (p.dense) return b * p.kv_len + pg * kPage;
        int phys = pg < p.width ? p.table[(int64_t)row * p.width + pg] : -1;
        if (phys < 0 || phys >= p.capacity) { sdl_raise(p.err, SDL_DEVERR_BAD_INDEX); phys = 0; }
        return (p.layer * p.capacity + phys) * kPage;
    };
    int tok_l = lane < my_n ? page_tok(lane) : 0;  // lane l: this warp's page l (then l + 32, ...)

    pdl_wait();

    // Q as B fragments: column grp of this warp, dims permuted as above.
    uint32_t qf[MT][2];
    {
        const int col = grp;
        const bool ok = col < ncol && col / p.ratio < nvalid;
        const T* qp = nullptr;
        if (ok) {
            const int j = col / p.ratio, h = g * p.ratio + col % p.ratio;
            qp = reinterpret_cast<const T*>(p.q) + b * p.q_sb + j * p.q_sj + h * p.q_sh;
        }
#pragma unroll
        for (int j = 0; j < KC; ++j)
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                qf[2 * j + h][0] = ok ? ld_u32(qp + 32 * j + 8 * tq + 4 * h) : 0u;
                qf[2 * j + h][1] = ok ? ld_u32(qp + 32 * j + 8 * tq + 4 * h + 2) : 0u;
            }
        if (ok && p.rope_cos != nullptr) {  // dims e and e + d/2 sit in pieces j and j + KC/2
            const int64_t ro = (int64_t)(b * p.chunk + col / p.ratio) * p.rope_stride;
            const T* cr = reinterpret_cast<const T*>(p.rope_cos) + ro;
            const T* sr = reinterpret_cast<const T*>(p.rope_sin) + ro;
#pragma unroll
            for (int j = 0; j < KC / 2; ++j)
#pragma unroll
                for (int h = 0; h < 2; ++h)
#pragma unroll
                    for (int r = 0; r < 2; ++r)
                        rope_u32<T>(qf[2 * j + h][r], qf[2 * (j + KC / 2) + h][r], cr, sr,
                                    32 * j + 8 * tq + 4 * h + 2 * r, HD / 2);
        }
    }
    int lim[2];
    float m_run[2], l_run[2];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
        const int col = 2 * tq + e;
        const int j = col / p.ratio;
        lim[e] = (col < ncol && j < nvalid) ? start + j + 1 : lmax;
        m_run[e] = -INFINITY;
        l_run[e] = 0.f;
    }
    const int lim_min = __reduce_min_sync(0xffffffffu, min(lim[0], lim[1]));
    float acc[MT][4];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int r = 0; r < 4; ++r) acc[mt][r] = 0.f;

    // Fused append: the warp that attends page pg first stores this kv
    // head's new rows that fall in it (lanes own 16-byte pieces, K then V);
    // __syncwarp orders those stores before the warp's own loads of the page.
    // With RoPE a K lane rotates its piece with the partner piece (dims +-
    // d/2; the piece count is a power of two) and the row's cos / sin.
    auto append_page = [&](int pg, int t0) {
        constexpr int PC = RB / 16;
        const int lo = max(start, pg * kPage), hi = min(start + nvalid, (pg + 1) * kPage);
        for (int pos = lo; pos < hi; ++pos) {
            const int64_t nrow = (int64_t)b * p.chunk + (pos - start);
            const int64_t src = nrow * p.new_stride + g * RB;
            const int64_t dst = (int64_t)(t0 + pos - pg * kPage) * rs + g * RB;
            if (lane < 2 * PC) {
                const bool isv = lane >= PC;
                const int c = lane % PC;
                const int cb = c * 16;
                const char* s0 = (isv ? p.v_new : p.k_new) + src;
                uint4 v = *reinterpret_cast<const uint4*>(s0 + cb);
                if (!isv && p.rope_cos != nullptr) {
                    const uint4 par = *reinterpret_cast<const uint4*>(s0 + (c ^ (PC / 2)) * 16);
                    const int64_t ro = nrow * p.rope_stride * (int64_t)sizeof(T) + cb;
                    const uint4 cv = *reinterpret_cast<const uint4*>(p.rope_cos + ro);
                    const uint4 sv = *reinterpret_cast<const uint4*>(p.rope_sin + ro);
                    v = rope_piece<T>(v, par, cv, sv, c < PC / 2);
                }
                *reinterpret_cast<uint4*>((isv ? p.v_pool : p.k_pool) + dst + cb) = v;
            }
        }
        __syncwarp();
    };
    uint4 kr[2][KC];  // key rows grp, grp + 8
    uint4 vr[4][VC];  // keys 2tq, 2tq + 1, 2tq + 8, 2tq + 9
    auto load_k = [&](int t0, int pos0) {
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const int key = grp + 8 * r;
            const bool ok = pos0 + key < klim;
            const char* src = p.k_src + (int64_t)(t0 + key) * rs + g * RB + tq * 16;
#pragma unroll
            for (int j = 0; j < KC; ++j)
                kr[r][j] = ok ? *reinterpret_cast<const uint4*>(src + j * 64) : make_uint4(0u, 0u, 0u, 0u);
        }
    };
    auto load_v = [&](int t0, int pos0) {
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const int key = 2 * tq + (r & 1) + 8 * (r >> 1);
            const bool ok = pos0 + key < klim;
            const char* src = p.v_src + (int64_t)(t0 + key) * rs + g * RB + grp * 16;
#pragma unroll
            for (int u = 0; u < VC; ++u)
                vr[r][u] = ok ? *reinterpret_cast<const uint4*>(src + u * 128) : make_uint4(0u, 0u, 0u, 0u);
        }
    };

    const bool p_split = p.out_dtype == SDL_F32;
    const bool append = p.k_new != nullptr;
    if (my_n > 0) {
        const int t0 = __shfl_sync(0xffffffffu, tok_l, 0);
        const int pg = pbeg + wi;
        if (append) append_page(pg, t0);
        load_k(t0, pg * kPage);
        load_v(t0, pg * kPage);
    }
    for (int k = 0; k < my_n; ++k) {
        const int pg = pbeg + wi + k * WH;
        // S^T[key][col] over this page's 16 keys
        float s[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int j = 0; j < KC; ++j) {
            uint32_t a0[4] = {u4_word<0>(kr[0][j]), u4_word<0>(kr[1][j]), u4_word<1>(kr[0][j]), u4_word<1>(kr[1][j])};
            mma_16816<T>(s, a0, qf[2 * j][0], qf[2 * j][1]);
            uint32_t a1[4] = {u4_word<2>(kr[0][j]), u4_word<2>(kr[1][j]), u4_word<3>(kr[0][j]), u4_word<3>(kr[1][j])};
            mma_16816<T>(s, a1, qf[2 * j + 1][0], qf[2 * j + 1][1]);
        }
        const bool more = k + 1 < my_n;
        int t_next = 0;
        if (more) {
            if (((k + 1) & 31) == 0) tok_l = k + 1 + lane < my_n ? page_tok(k + 1 + lane) : 0;
            t_next = __shfl_sync(0xffffffffu, tok_l, (k + 1) & 31);
            if (append) append_page(pg + WH, t_next);
            load_k(t_next, (pg + WH) * kPage);
        }

        // Online softmax per query column, log2 domain, lazy running max
        // (m_run moves only when a page's max exceeds it by 2^kLazyLog2).
        const int pos_lo = pg * kPage + grp, pos_hi = pos_lo + 8;
        const bool whole = (pg + 1) * kPage <= lim_min;
        float mx[2];
        bool need = false;
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            if (!whole) {
                if (pos_lo >= lim[e]) s[e] = -INFINITY;
                if (pos_hi >= lim[e]) s[2 + e] = -INFINITY;
            }
            float m = fmaxf(s[e], s[2 + e]);
            m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 4));
            m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 8));
            m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 16));
            mx[e] = m * p.scale_log2;
            need |= mx[e] > m_run[e] + kLazyLog2;
        }
        if (__any_sync(0xffffffffu, need)) {
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                if (!(mx[e] > m_run[e] + kLazyLog2)) continue;
                const float alpha = ex2_approx(m_run[e] - mx[e]);  // 0 on the first page
                m_run[e] = mx[e];
                l_run[e] *= alpha;
#pragma unroll
                for (int mt = 0; mt < MT; ++mt) {
                    acc[mt][e] *= alpha;
                    acc[mt][2 + e] *= alpha;
                }
            }
        }
        float pv[4];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            const float muse = m_run[e] == -INFINITY ? 0.f : m_run[e];
            pv[e] = ex2_approx(fmaf(s[e], p.scale_log2, -muse));
            pv[2 + e] = ex2_approx(fmaf(s[2 + e], p.scale_log2, -muse));
            l_run[e] += pv[e] + pv[2 + e];
        }
        // P^T as B fragments: keys 2c, 2c+1 (and 2c+8, 2c+9) of column g.
        const uint32_t pb0 = movmatrix_trans(pack2<T>(pv[0], pv[1]));
        const uint32_t pb1 = movmatrix_trans(pack2<T>(pv[2], pv[3]));
        uint32_t pl0 = 0u, pl1 = 0u;
        if (p_split) {
            pl0 = movmatrix_trans(pack2<T>(pv[0] - round_trip<T>(pv[0]), pv[1] - round_trip<T>(pv[1])));
            pl1 = movmatrix_trans(pack2<T>(pv[2] - round_trip<T>(pv[2]), pv[3] - round_trip<T>(pv[3])));
        }

        // O^T[dim][col] += sum_key V[key][dim] P^T[key][col]
#pragma unroll
        for (int u = 0; u < VC; ++u) {
#define SDL_DIRECT_PV(W)                                                                             \
    {                                                                                                \
        const uint32_t x0 = u4_word<W>(vr[0][u]), x1 = u4_word<W>(vr[1][u]);                         \
        const uint32_t x2 = u4_word<W>(vr[2][u]), x3 = u4_word<W>(vr[3][u]);                         \
        uint32_t a[4] = {__byte_perm(x0, x1, 0x5410), __byte_perm(x0, x1, 0x7632),                   \
                         __byte_perm(x2, x3, 0x5410), __byte_perm(x2, x3, 0x7632)};                  \
        mma_16816<T>(acc[4 * u + W], a, pb0, pb1);                                                   \
        if (p_split) mma_16816<T>(acc[4 * u + W], a, pl0, pl1);                                      \
    }
            SDL_DIRECT_PV(0)
            SDL_DIRECT_PV(1)
            SDL_DIRECT_PV(2)
            SDL_DIRECT_PV(3)
#undef SDL_DIRECT_PV
        }
        if (more) load_v(t_next, (pg + WH) * kPage);
    }
    pdl_launch_dependents();  // the split merge may be scheduled during the epilogue

    // Each warp's (m, l, O) to shared memory, columns 2tq + e.
#pragma unroll
    for (int e = 0; e < 2; ++e) {
        float l = l_run[e];
        l += __shfl_xor_sync(0xffffffffu, l, 4);
        l += __shfl_xor_sync(0xffffffffu, l, 8);
        l += __shfl_xor_sync(0xffffffffu, l, 16);
        const int col = 2 * tq + e;
        if (grp == 0) {
            s_m[warp][col] = m_run[e];
            s_l[warp][col] = l;
        }
#pragma unroll
        for (int u = 0; u < VC; ++u)
#pragma unroll
            for (int w = 0; w < 4; ++w)
                *reinterpret_cast<float2*>(&s_part[warp][col][64 * u + 8 * grp + 2 * w]) =
                    make_float2(acc[4 * u + w][e], acc[4 * u + w][2 + e]);
    }
    __syncthreads();

    // Merge each head's warps: thread -> (head, column, 4 head dims).  A
    // column with a key in this split saw it in the first page of the
    // head's warp wi = 0, so M is finite.
    constexpr int NQ = HD / 4;
    for (int idx = threadIdx.x; idx < G * kDirCols * NQ; idx += kDirWarps * 32) {
        const int hg = idx / (kDirCols * NQ);
        const int col = (idx / NQ) % kDirCols, d0 = (idx % NQ) * 4;
        if (col >= ncol) continue;
        const int j = col / p.ratio;
        if (j >= nvalid) continue;
        const int L = start + j + 1;
        const int np_c = (L + kPage - 1) / kPage;
        if (pbeg >= np_c) continue;
        const int ns_c = (np_c + p.pps - 1) / p.pps;
        float M = -INFINITY;
        for (int w = hg; w < kDirWarps; w += G) M = fmaxf(M, s_m[w][col]);
        float den = 0.f;
        float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int w = hg; w < kDirWarps; w += G) {
            const float mw = s_m[w][col];
            if (mw == -INFINITY) continue;  // a warp with no key of this column
            const float wt = ex2_approx(mw - M);
            den = fmaf(wt, s_l[w][col], den);
            const float4 v = *reinterpret_cast<const float4*>(&s_part[w][col][d0]);
            o.x = fmaf(wt, v.x, o.x); o.y = fmaf(wt, v.y, o.y);
            o.z = fmaf(wt, v.z, o.z); o.w = fmaf(wt, v.w, o.w);
        }
        const int h = (blockIdx.y * G + hg) * p.ratio + col % p.ratio;
        if (ns_c == 1) {
            const float inv = 1.f / den;
            const int64_t ob = b * p.o_sb + j * p.o_sj + h * p.o_sh + d0;
            store_from_f32(p.out, ob, p.out_dtype, o.x * inv);
            store_from_f32(p.out, ob + 1, p.out_dtype, o.y * inv);
            store_from_f32(p.out, ob + 2, p.out_dtype, o.z * inv);
            store_from_f32(p.out, ob + 3, p.out_dtype, o.w * inv);
        } else {
            const int64_t pidx = (((int64_t)b * p.nsplit + split) * p.chunk + j) * p.Hq + h;
            *reinterpret_cast<float4*>(p.o_part + pidx * HD + d0) = o;
            if (d0 == 0) {
                p.ml_part[pidx * 2] = M;
                p.ml_part[pidx * 2 + 1] = den;
            }
        }
    }
}

// Merge split-K partials (m in log2 units, unnormalised O, l).  One warp per
// (sequence, chunk row, q head), each lane owning 4 consecutive head dims.
// The merge is latency bound: up to kCombineOneRound splits take one round
// of loads (every split's m, l and partial row at once); more take two
// dependent rounds, the splits' (m, l) pairs (lane s holds split s, reduced
// by an online max/sum across lanes), then 16 partial rows at a time.
__global__ void __launch_bounds__(128) attn_combine_kernel(TcParams p, int hd) {
    if (p.overlap) pdl_launch_dependents();  // layers back to back: the next attention may become resident
    pdl_wait();  // partials come from the attention launch just before
    pdl_launch_dependents();  // the next launch may become resident; it waits for this grid to finish
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
    const int ns = min(p.nsplit, (np_c + p.pps - 1) / p.pps);
    if (ns <= 1) return;
    const int64_t idx0 = (((int64_t)b * p.nsplit) * p.chunk + j) * p.Hq + h;
    const int64_t sstride = (int64_t)p.chunk * p.Hq;
    const int64_t ob = b * p.o_sb + j * p.o_sj + h * p.o_sh;
    // Every split below ns saw at least one key of this row, so each m is finite.
    if (ns <= kCombineOneRound && hd <= 128) {
        // One round of loads: every split's (m, l) (the same addresses in
        // every lane) and this lane's 4 head dims of every split's row.
        const int d0 = lane * 4;
        const bool mine = d0 < hd;
        float2 ml[kCombineOneRound];
        float4 o[kCombineOneRound];
#pragma unroll
        for (int t = 0; t < kCombineOneRound; ++t) {
            ml[t] = make_float2(-INFINITY, 0.f);
            o[t] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (t < ns) {
                const int64_t idx = idx0 + t * sstride;
                ml[t] = *reinterpret_cast<const float2*>(p.ml_part + idx * 2);
                if (mine) o[t] = *reinterpret_cast<const float4*>(p.o_part + idx * hd + d0);
            }
        }
        float M = -INFINITY;
#pragma unroll
        for (int t = 0; t < kCombineOneRound; ++t) M = fmaxf(M, ml[t].x);
        float den = 0.f;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int t = 0; t < kCombineOneRound; ++t) {
            const float w = ex2_approx(ml[t].x - M);  // 0 for the padding slots
            den = fmaf(w, ml[t].y, den);
            acc.x = fmaf(w, o[t].x, acc.x);
            acc.y = fmaf(w, o[t].y, acc.y);
            acc.z = fmaf(w, o[t].z, acc.z);
            acc.w = fmaf(w, o[t].w, acc.w);
        }
        if (mine) {
            const float inv = 1.f / den;
            store_from_f32(p.out, ob + d0, p.out_dtype, acc.x * inv);
            store_from_f32(p.out, ob + d0 + 1, p.out_dtype, acc.y * inv);
            store_from_f32(p.out, ob + d0 + 2, p.out_dtype, acc.z * inv);
            store_from_f32(p.out, ob + d0 + 3, p.out_dtype, acc.w * inv);
        }
        return;
    }
    float M = -INFINITY, den = 0.f;
    for (int s = lane; s < ns; s += 32) {
        const float2 ml = *reinterpret_cast<const float2*>(p.ml_part + (idx0 + s * sstride) * 2);
        const float mn = fmaxf(M, ml.x);
        den = den * ex2_approx(M - mn) + ml.y * ex2_approx(ml.x - mn);
        M = mn;
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        const float M2 = __shfl_xor_sync(0xffffffffu, M, off);
        const float d2 = __shfl_xor_sync(0xffffffffu, den, off);
        const float mn = fmaxf(M, M2);
        den = (M == -INFINITY ? 0.f : den * ex2_approx(M - mn)) + (M2 == -INFINITY ? 0.f : d2 * ex2_approx(M2 - mn));
        M = mn;
    }
    const float inv = 1.f / den;
    for (int d0 = lane * 4; d0 < hd; d0 += 128) {
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int s = 0; s < ns; s += 16) {
            float w[16];
            float4 o[16];
#pragma unroll
            for (int t = 0; t < 16; ++t) {
                w[t] = -INFINITY;
                o[t] = make_float4(0.f, 0.f, 0.f, 0.f);
                if (s + t < ns) {
                    const int64_t idx = idx0 + (s + t) * sstride;
                    w[t] = p.ml_part[idx * 2];
                    o[t] = *reinterpret_cast<const float4*>(p.o_part + idx * hd + d0);
                }
            }
#pragma unroll
            for (int t = 0; t < 16; ++t) {
                const float wt = ex2_approx(w[t] - M);  // 0 for the padding slots
                acc.x = fmaf(wt, o[t].x, acc.x);
                acc.y = fmaf(wt, o[t].y, acc.y);
                acc.z = fmaf(wt, o[t].z, acc.z);
                acc.w = fmaf(wt, o[t].w, acc.w);
            }
        }
        store_from_f32(p.out, ob + d0, p.out_dtype, acc.x * inv);
        store_from_f32(p.out, ob + d0 + 1, p.out_dtype, acc.y * inv);
        store_from_f32(p.out, ob + d0 + 2, p.out_dtype, acc.z * inv);
        store_from_f32(p.out, ob + d0 + 3, p.out_dtype, acc.w * inv);
    }
}

// ---------------------------------------------- rows-on-M mma.sync kernel
// attn_rows_kernel: paged attention for blocks of query rows -- the
// (gamma+1)-token verify block and prefill chunks -- in the FlashAttention-2
// register layout.  Row r = token j * ratio + head offset (the GQA rows of
// one kv head); a warp owns 16 rows on the MMA M dimension and walks 32-key
// tiles:
//   S[16 x 32] = Q K^T   Q fragments held in registers, K by ldmatrix;
//   P = 2^(S * scale * log2(e) - m) per row: the row max takes two quad
//       shuffles, and O and l are rescaled only when it grows by more than
//       2^kLazyLog2 (so P <= 2^kLazyLog2);
//   O[16 x d] += P V     the S accumulators re-packed in place as the A
//       operand (no transposes), V by ldmatrix.trans.
// Against the keys-on-M kernel above this needs about a fifth of the
// instructions per key and row, which is what verify blocks are bound by.
// A producer warp streams tiles of two 16-token pages of K and V (2 KB
// 128-byte-swizzled boxes) through a TMA ring, first storing the call's new
// K/V rows that fall in its pages (fused append), as attn_tc_kernel does.
// CTA = (split, row tile x kv head, sequence); rows whose pages span several
// splits leave fp32 partials (same layout) for attn_combine_kernel.
constexpr int kRowWarps = 4;                 // consumer warps of a full row tile
constexpr int kRowTile = 16 * kRowWarps;     // query rows per CTA
constexpr int kTilePages = 2;                // 16-token pages per ring stage (32-key tiles)
constexpr int kRowStages = 4;                // ring depth

template <int HD>
constexpr int rows_stage_bytes() { return kTilePages * 2 * (HD / 64) * kBoxBytes; }

template <int HD, typename T>
__global__ void __launch_bounds__((kRowWarps + 1) * 32, 2)
attn_rows_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv, const TcParams p) {
    constexpr int DO = HD / 64;
    constexpr int KS = HD / 16;                   // k-steps of S = Q K^T
    constexpr int ON = HD / 8;                    // n-tiles (8 head dims) of O
    constexpr int SN = kTilePages * kPage / 8;    // n-tiles (8 keys) of S
    constexpr int PAGE_BYTES = 2 * DO * kBoxBytes;
    constexpr int STAGE_BYTES = rows_stage_bytes<HD>();
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int NS = p.stages;  // ring depth (the plan's; kRowStages)
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + NS * STAGE_BYTES);
    uint64_t* empty = full + NS;
    __shared__ int s_abort_flag;
    volatile int* s_abort = &s_abort_flag;

    if (p.overlap) pdl_launch_dependents();  // the next layer's launch may become resident now
    const int b = blockIdx.z, split = blockIdx.x;
    const int g = blockIdx.y % p.Hkv, rt = blockIdx.y / p.Hkv;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ncons = (int)(blockDim.x >> 5) - 1;
    const int R = p.chunk * p.ratio;

    // Row metadata and the first page-table batch are read before
    // griddepcontrol.wait, under the same rule as attn_tc_kernel; Q, the new
    // K/V rows and the pool pages only after it.
    const int start = p.starts[b];
    const int nvalid = p.valid_rows ? min(p.valid_rows[b], p.chunk) : p.chunk;
    const int r_lo = rt * kRowTile;
    const int r_hi = min(R, r_lo + kRowTile);
    int lmax = 0;
    if (r_lo < R && r_lo / p.ratio < nvalid) lmax = start + min((r_hi - 1) / p.ratio, nvalid - 1) + 1;
    const int npages = lmax > 0 ? (lmax + kPage - 1) / kPage : 0;
    const int pbeg = split * p.pps;  // pps is a multiple of kTilePages
    const int pend = min(npages, pbeg + p.pps);
    // A span past the grid (max_limit below some starts[b] + chunk) is
    // reported and its excess pages are not attended.
    if ((npages + p.pps - 1) / p.pps > p.nsplit && threadIdx.x == 0 && split == 0)
        sdl_raise(p.err, SDL_DEVERR_BAD_INDEX);
    if (lmax <= 0 || pbeg >= pend) return;
    const int np = pend - pbeg;
    const int ntile = (np + kTilePages - 1) / kTilePages;
    const int row = p.dense ? 0 : p.rows[b];
    // Pool token row of page pg (out-of-range entries raise and read row 0).
    auto page_tok = [&](int pg) -> int {
        if (p.dense) return b * p.kv_len + pg * kPage;
        int phys = pg < p.width ? p.table[(int64_t)row * p.width + pg] : -1;
        if (phys < 0 || phys >= p.capacity) { sdl_raise(p.err, SDL_DEVERR_BAD_INDEX); phys = 0; }
        return (p.layer * p.capacity + phys) * kPage;
    };
    const int tok_first = (warp == ncons && lane < np) ? page_tok(pbeg + lane) : 0;

    if (threadIdx.x == 0) {
        *s_abort = 0;
        for (int s = 0; s < NS; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], ncons);
        }
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == ncons) {
        // ------------------------------------------------------- producer
        if (lane == 0) { prefetch_tmap(&tmk); prefetch_tmap(&tmv); }
        // first page of this split that holds a new row (-1: no append)
        const int app_page = p.k_new != nullptr && max(pbeg, start / kPage) < pend ? max(pbeg, start / kPage) : -1;
        // Layers back to back (p.overlap) with the fused append: tiles wholly
        // before the first new row's page hold keys of earlier, completed
        // launches, and the first ring stages of them are issued before
        // griddepcontrol.wait (as in attn_tc_kernel).
        const int npre = p.overlap && p.k_new != nullptr
                             ? min(NS, min(ntile, max(0, (start / kPage - pbeg) / kTilePages))) : 0;
        for (int i = 0; i < npre; ++i) {
            const int k = i * kTilePages;
            const int cnt0 = min(32, np);
            int tq[kTilePages];
#pragma unroll
            for (int q = 0; q < kTilePages; ++q) tq[q] = __shfl_sync(0xffffffffu, tok_first, min(k + q, cnt0 - 1));
            if (lane == 0) {
                mbar_arrive_expect_tx(&full[i], STAGE_BYTES);
                uint8_t* sbuf = smem + i * STAGE_BYTES;
#pragma unroll
                for (int q = 0; q < kTilePages; ++q) {
#pragma unroll
                    for (int dd = 0; dd < DO; ++dd) {
                        tma_load_4d(sbuf + q * PAGE_BYTES + dd * kBoxBytes, &tmk, &full[i], 0, dd, g, tq[q]);
                        tma_load_4d(sbuf + q * PAGE_BYTES + (DO + dd) * kBoxBytes, &tmv, &full[i], 0, dd, g,
                                    tq[q]);
                    }
                }
            }
            __syncwarp();
        }
        pdl_wait();
        // Fused append of kv head g's slice of every new row whose page lies
        // in [pbeg, pend), before the tile holding the first of them is issued.
        auto append_rows = [&]() {
            const int row_bytes = p.Hkv * HD * (int)sizeof(T);
            const int hoff = g * HD * (int)sizeof(T);
            for (int j0 = 0; j0 < nvalid; j0 += kAppendBatch) {
                int64_t trow = -1;
                if (lane < kAppendBatch && j0 + lane < nvalid) {
                    const int pos = start + j0 + lane, pg = pos / kPage;
                    if (pg >= pbeg && pg < pend) {
                        const int phys = pg < p.width ? p.table[(int64_t)row * p.width + pg] : -1;
                        if (phys < 0 || phys >= p.capacity) sdl_raise(p.err, SDL_DEVERR_BAD_INDEX);
                        else trow = (int64_t)(p.layer * p.capacity + phys) * kPage + pos % kPage;
                    }
                }
                int64_t src[kAppendBatch], dst[kAppendBatch];
                int nrow[kAppendBatch];
#pragma unroll
                for (int u = 0; u < kAppendBatch; ++u) {
                    const int64_t tr = __shfl_sync(0xffffffffu, trow, u);
                    nrow[u] = b * p.chunk + j0 + u;
                    src[u] = (int64_t)nrow[u] * p.new_stride + hoff;
                    dst[u] = tr >= 0 ? tr * row_bytes + hoff : -1;
                }
                copy_new_rows<HD, T>(p, lane, src, dst, nrow, min(kAppendBatch, nvalid - j0));
            }
            asm volatile("fence.proxy.async.global;" ::: "memory");
            __syncwarp();
        };
        int issued = 0;
        bool stop = false;
        for (int i0 = 0; i0 < np && !stop; i0 += 32) {  // 32 pages (16 tiles) per table batch
            const int tok = i0 == 0 ? tok_first : (i0 + lane < np ? page_tok(pbeg + i0 + lane) : 0);
            const int cnt = min(32, np - i0);
            for (int k = 0; k < cnt; k += kTilePages) {
                const int i = (i0 + k) / kTilePages;
                const int st = i % NS;
                // a ragged last tile (the split's last pages) repeats its last
                // page: the repeats' keys lie past every row's limit and are
                // masked (non-final splits hold whole tiles: pps is aligned)
                int tq[kTilePages];
#pragma unroll
                for (int q = 0; q < kTilePages; ++q) tq[q] = __shfl_sync(0xffffffffu, tok, min(k + q, cnt - 1));
                const int pg0 = pbeg + i0 + k;
                if (i < npre) { issued = i + 1; continue; }  // issued before the wait
                if (app_page >= pg0 && app_page < pg0 + kTilePages) append_rows();  // app_page < pend
                if (i >= NS) {
                    int ok = 1;
                    if (lane == 0) ok = mbar_wait_bounded(&empty[st], ((i / NS) - 1) & 1, kWaitLimit) ? 1 : 0;
                    ok = __shfl_sync(0xffffffffu, ok, 0);
                    if (!ok || *s_abort) {
                        if (lane == 0 && !ok) { sdl_raise(p.err, SDL_DEVERR_TIMEOUT); *s_abort = 1; }
                        stop = true;
                        break;
                    }
                }
                if (lane == 0) {
                    mbar_arrive_expect_tx(&full[st], STAGE_BYTES);
                    uint8_t* sbuf = smem + st * STAGE_BYTES;
#pragma unroll
                    for (int q = 0; q < kTilePages; ++q) {
#pragma unroll
                        for (int dd = 0; dd < DO; ++dd) {
                            tma_load_4d(sbuf + q * PAGE_BYTES + dd * kBoxBytes, &tmk, &full[st], 0, dd, g, tq[q]);
                            tma_load_4d(sbuf + q * PAGE_BYTES + (DO + dd) * kBoxBytes, &tmv, &full[st], 0, dd, g,
                                        tq[q]);
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
            for (int i = max(0, issued - NS); i < issued; ++i)
                (void)mbar_wait_bounded(&full[i % NS], (i / NS) & 1, kWaitLimit);
        }
        pdl_launch_dependents();
        return;
    }

    // ----------------------------------------------------------- consumers
    pdl_wait();  // Q comes from the preceding kernels
    const int t4 = lane & 3, gq = lane >> 2;
    const int r0 = r_lo + warp * 16;
    const int ra = r0 + gq, rb = ra + 8;
    const int ja = ra / p.ratio, jb = rb / p.ratio;
    const bool va = ra < r_hi && ja < nvalid, vb = rb < r_hi && jb < nvalid;
    const bool active = r0 < r_hi && r0 / p.ratio < nvalid;  // rows ascend: the warp's first row decides
    // key limits (rows that are not attended get the tile's limit: finite values, never stored)
    const int lim_a = va ? start + ja + 1 : lmax, lim_b = vb ? start + jb + 1 : lmax;
    const int lim_min = __reduce_min_sync(0xffffffffu, min(lim_a, lim_b));

    uint32_t qa[KS][4];
    {
        const T* q0 = reinterpret_cast<const T*>(p.q) + b * p.q_sb;
        const T* qpa = q0 + ja * p.q_sj + (g * p.ratio + ra % p.ratio) * p.q_sh;
        const T* qpb = q0 + jb * p.q_sj + (g * p.ratio + rb % p.ratio) * p.q_sh;
#pragma unroll
        for (int ks = 0; ks < KS; ++ks) {
            qa[ks][0] = va ? ld_u32(qpa + ks * 16 + 2 * t4) : 0u;
            qa[ks][1] = vb ? ld_u32(qpb + ks * 16 + 2 * t4) : 0u;
            qa[ks][2] = va ? ld_u32(qpa + ks * 16 + 8 + 2 * t4) : 0u;
            qa[ks][3] = vb ? ld_u32(qpb + ks * 16 + 8 + 2 * t4) : 0u;
        }
        if (p.rope_cos != nullptr) {  // dims e and e + d/2 sit in k-steps ks and ks + KS/2
#pragma unroll
            for (int hr = 0; hr < 2; ++hr) {
                if (!(hr ? vb : va)) continue;
                const int64_t ro = (int64_t)(b * p.chunk + (hr ? jb : ja)) * p.rope_stride;
                const T* cr = reinterpret_cast<const T*>(p.rope_cos) + ro;
                const T* sr = reinterpret_cast<const T*>(p.rope_sin) + ro;
#pragma unroll
                for (int ks = 0; ks < KS / 2; ++ks) {
                    rope_u32<T>(qa[ks][hr], qa[ks + KS / 2][hr], cr, sr, ks * 16 + 2 * t4, HD / 2);
                    rope_u32<T>(qa[ks][2 + hr], qa[ks + KS / 2][2 + hr], cr, sr, ks * 16 + 8 + 2 * t4, HD / 2);
                }
            }
        }
    }
    float o[ON][4];
#pragma unroll
    for (int dn = 0; dn < ON; ++dn)
#pragma unroll
        for (int e = 0; e < 4; ++e) o[dn][e] = 0.f;
    float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.f, l_b = 0.f;

    // ldmatrix lane offsets inside a stage (128-byte swizzle: 16-byte chunk
    // c of token row t sits at chunk c ^ (t & 7); here t & 7 = lane & 7).
    // K (S's B operand): matrix m = lane / 8 holds keys 8 nt + (lane & 7),
    // head-dim chunk 2 ks + m (two k-steps per x4).  V (P V's B operand,
    // transposed): keys 16 kk + 8 (m & 1) + (lane & 7), dim chunk dn + m / 2.
    const int sw = lane & 7, mq = lane >> 3;
    uint32_t kofs[SN];
#pragma unroll
    for (int nt = 0; nt < SN; ++nt) kofs[nt] = (nt >> 1) * PAGE_BYTES + ((nt & 1) * 8 + sw) * 128;
    const uint32_t vrow = ((mq & 1) * 8 + sw) * 128;
    const int vch = mq >> 1;
    const bool p_split = p.out_dtype == SDL_F32;
    const uint32_t sbase = smem_u32(smem);
    bool aborted = false;

    for (int i = 0; i < ntile; ++i) {
        const int st = i % NS;
        const bool ok = __all_sync(0xffffffffu, mbar_wait_bounded(&full[st], (i / NS) & 1, kWaitLimit));
        if (!ok) {
            if (lane == 0) { sdl_raise(p.err, SDL_DEVERR_TIMEOUT); *s_abort = 1; }
            aborted = true;
            break;
        }
        if (active) {
            const uint32_t sb = sbase + st * STAGE_BYTES;
            float s[SN][4];
#pragma unroll
            for (int nt = 0; nt < SN; ++nt)
#pragma unroll
                for (int e = 0; e < 4; ++e) s[nt][e] = 0.f;
#pragma unroll
            for (int ks = 0; ks < KS; ks += 2) {
                const int c = 2 * ks + mq;
                const uint32_t co = (c >> 3) * kBoxBytes + (((c & 7) ^ sw) << 4);
#pragma unroll
                for (int nt = 0; nt < SN; ++nt) {
                    uint32_t b0, b1, b2, b3;
                    ldmatrix_x4(sb + kofs[nt] + co, b0, b1, b2, b3);
                    mma_16816<T>(s[nt], qa[ks], b0, b1);
                    mma_16816<T>(s[nt], qa[ks + 1], b2, b3);
                }
            }
            // causal mask (tiles wholly below every row's limit skip it) and row maxima
            const int pos0 = (pbeg + i * kTilePages) * kPage;
            const bool whole = pos0 + kTilePages * kPage <= lim_min;
            float mxa = -INFINITY, mxb = -INFINITY;
#pragma unroll
            for (int nt = 0; nt < SN; ++nt)
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    if (!whole) {
                        const int key = pos0 + nt * 8 + 2 * t4 + e;
                        if (key >= lim_a) s[nt][e] = -INFINITY;
                        if (key >= lim_b) s[nt][2 + e] = -INFINITY;
                    }
                    mxa = fmaxf(mxa, s[nt][e]);
                    mxb = fmaxf(mxb, s[nt][2 + e]);
                }
            mxa = fmaxf(mxa, __shfl_xor_sync(0xffffffffu, mxa, 1));
            mxa = fmaxf(mxa, __shfl_xor_sync(0xffffffffu, mxa, 2));
            mxb = fmaxf(mxb, __shfl_xor_sync(0xffffffffu, mxb, 1));
            mxb = fmaxf(mxb, __shfl_xor_sync(0xffffffffu, mxb, 2));
            mxa *= p.scale_log2;
            mxb *= p.scale_log2;
            const bool na = mxa > m_a + kLazyLog2, nb = mxb > m_b + kLazyLog2;
            if (__any_sync(0xffffffffu, na || nb)) {
                if (na) {
                    const float alpha = ex2_approx(m_a - mxa);  // 0 on the first keys
                    m_a = mxa;
                    l_a *= alpha;
#pragma unroll
                    for (int dn = 0; dn < ON; ++dn) { o[dn][0] *= alpha; o[dn][1] *= alpha; }
                }
                if (nb) {
                    const float alpha = ex2_approx(m_b - mxb);
                    m_b = mxb;
                    l_b *= alpha;
#pragma unroll
                    for (int dn = 0; dn < ON; ++dn) { o[dn][2] *= alpha; o[dn][3] *= alpha; }
                }
            }
            // P as the A operand of P V: k-step kk takes S n-tiles 2 kk (keys
            // 2t, 2t+1 of rows g, g+8) and 2 kk + 1 (keys 8 + 2t, 9 + 2t)
            const float ua = m_a == -INFINITY ? 0.f : m_a, ub = m_b == -INFINITY ? 0.f : m_b;
            uint32_t pa[SN / 2][4], pl[SN / 2][4];
#pragma unroll
            for (int nt = 0; nt < SN; ++nt) {
                const float p0 = ex2_approx(fmaf(s[nt][0], p.scale_log2, -ua));
                const float p1 = ex2_approx(fmaf(s[nt][1], p.scale_log2, -ua));
                const float p2 = ex2_approx(fmaf(s[nt][2], p.scale_log2, -ub));
                const float p3 = ex2_approx(fmaf(s[nt][3], p.scale_log2, -ub));
                l_a += p0 + p1;
                l_b += p2 + p3;
                const int kk = nt >> 1, hf = (nt & 1) * 2;
                pa[kk][hf] = pack2<T>(p0, p1);
                pa[kk][hf + 1] = pack2<T>(p2, p3);
                if (p_split) {
                    pl[kk][hf] = pack2<T>(p0 - round_trip<T>(p0), p1 - round_trip<T>(p1));
                    pl[kk][hf + 1] = pack2<T>(p2 - round_trip<T>(p2), p3 - round_trip<T>(p3));
                }
            }
#pragma unroll
            for (int kk = 0; kk < SN / 2; ++kk) {
#pragma unroll
                for (int dn = 0; dn < ON; dn += 2) {
                    const int c = dn + vch;
                    uint32_t v0, v1, v2, v3;
                    ldmatrix_x4_trans(sb + kk * PAGE_BYTES + (DO + (c >> 3)) * kBoxBytes + vrow + (((c & 7) ^ sw) << 4),
                                      v0, v1, v2, v3);
                    mma_16816<T>(o[dn], pa[kk], v0, v1);
                    mma_16816<T>(o[dn + 1], pa[kk], v2, v3);
                    if (p_split) {
                        mma_16816<T>(o[dn], pl[kk], v0, v1);
                        mma_16816<T>(o[dn + 1], pl[kk], v2, v3);
                    }
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[st]);
    }
    __syncthreads();
    pdl_launch_dependents();  // the split merge may be scheduled during the epilogue
    if (aborted || *s_abort || !active) return;

    // Epilogue: rows whose keys all lie in this split write the output,
    // split rows write partials.
    l_a += __shfl_xor_sync(0xffffffffu, l_a, 1);
    l_a += __shfl_xor_sync(0xffffffffu, l_a, 2);
    l_b += __shfl_xor_sync(0xffffffffu, l_b, 1);
    l_b += __shfl_xor_sync(0xffffffffu, l_b, 2);
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
        const bool v = hr ? vb : va;
        if (!v) continue;
        const int r = hr ? rb : ra;
        const int j = hr ? jb : ja;
        const int h = g * p.ratio + r % p.ratio;
        const int np_c = (start + j + 1 + kPage - 1) / kPage;
        if (pbeg >= np_c) continue;  // no key of this row in this split
        const float l = hr ? l_b : l_a;
        const int ns_c = (np_c + p.pps - 1) / p.pps;
        if (ns_c == 1) {
            const float inv = 1.f / l;
            const int64_t ob = b * p.o_sb + j * p.o_sj + h * p.o_sh + 2 * t4;
#pragma unroll
            for (int dn = 0; dn < ON; ++dn) {
                store_from_f32(p.out, ob + dn * 8, p.out_dtype, o[dn][2 * hr] * inv);
                store_from_f32(p.out, ob + dn * 8 + 1, p.out_dtype, o[dn][2 * hr + 1] * inv);
            }
        } else {
            const int64_t idx = (((int64_t)b * p.nsplit + split) * p.chunk + j) * p.Hq + h;
            float* op = p.o_part + idx * HD + 2 * t4;
#pragma unroll
            for (int dn = 0; dn < ON; ++dn)
                *reinterpret_cast<float2*>(op + dn * 8) = make_float2(o[dn][2 * hr], o[dn][2 * hr + 1]);
            if (t4 == 0) *reinterpret_cast<float2*>(p.ml_part + idx * 2) = make_float2(hr ? m_b : m_a, l);
        }
    }
}

// ------------------------------------------------------ tcgen05 verify path
// attn_sk_kernel: paged attention for blocks of up to 64 query rows per kv
// head (decode and the (gamma+1)-row verify) on the 5th-generation tensor
// cores, as a persistent stream-K kernel: the (sequence, kv head) pairs are
// laid end to end as 64-token tiles and every CTA (one per SM) takes an
// equal share of that tile sequence, so the grid is one balanced wave.  A
// CTA walks its share as segments (the part of one pair's tiles it owns)
// without draining its pipeline between them.  6 warps:
//   warp 4     producer: TMA of 64-token K/V tiles (4 pages, 2 KB boxes, one
//              lane per box) into a ring laid out as the canonical 128-byte
//              swizzled K-major (K) / MN-major (V) operand layouts; page-table
//              lookups run 32 tiles ahead;
//   warp 5     owns TMEM (512 columns); one thread issues tcgen05.mma (M = 64):
//              S[64 x 64] = Q[64 x d] K^T into a double-buffered TMEM tile,
//              then O[64 x d] += P_hi V + P_lo V into a TMEM accumulator that
//              alternates between two buffers from one segment to the next;
//   warps 0-3  softmax: query row m = 16*w + (lane % 16) (row m = j * ratio
//              + head offset; rows >= chunk*ratio are zero padding) lives in
//              TMEM lane 32*w + m % 16; lanes l and l + 16 hold the two
//              32-column halves of the row's S tile (16x32bx2 loads) and
//              share its max and sum by one shuffle.  Online softmax in the
//              log2 domain with a lazy rescale (O and l are rescaled in TMEM
//              only when the row max grows by more than 2^8); P is written as
//              a bf16/f16 hi+lo pair into swizzled shared memory.  They also
//              stage the next segment's Q (double buffered, cp.async issued at
//              a segment's start and published after its first tile) and run
//              each segment's epilogue: the final rows when the CTA owns the
//              whole pair, else fp32 partials (m in log2 units, unnormalised
//              O, l) that attn_sk_combine_kernel merges.
// Every mbarrier wait is bounded; on expiry the CTA records
// SDL_DEVERR_TIMEOUT, stops issuing, lets issued copies and MMAs land, and
// releases TMEM before exiting.
constexpr int kUTok = 64;             // tokens per tile
constexpr int kUPages = kUTok / kPage;
constexpr int kURows = 64;            // MMA M: padded query rows of one kv head
constexpr int kUThreads = 192;
constexpr int kUProducer = 4, kUMma = 5;
constexpr uint32_t kUTmemCols = 512;  // S double buffer (2 x 64 columns) + O double buffer (2 x 128)
constexpr int kUOCol = 2 * kUTok;     // TMEM column of O buffer 0; buffer 1 is 128 columns on
constexpr int kSkMaxPairs = 512;      // (sequence, kv head) pairs one launch may hold
constexpr int kSkMaxSeqs = 512;       // sequences one launch may hold
constexpr int kUmmaAutoMinKeys = 4096; // automatic plans: mean keys per sequence from which blocks use tcgen05
constexpr int kUmmaAutoMinRows = 48;   // ... and query rows per kv head
constexpr uint32_t kPollLimit = 1u << 24;  // idle polls (32 ns apart) of the tcgen05 MMA thread before a timeout

template <int HD>
struct USmem {
    static constexpr int DO = HD / 64;
    static constexpr int kNst = HD == 128 ? 5 : 8;  // K/V ring depth (fills the shared memory left)
    static constexpr int kQ = DO * kURows * 128;    // the Q buffer (8 KB per 64-column half)
    static constexpr int kHalf = kUTok * 128;       // one 64-column half of a K or V tile
    static constexpr int kStage = 2 * DO * kHalf;   // K halves then V halves
    static constexpr int kP = kURows * 128;         // one 64 x 64 16-bit P matrix
    static constexpr int kOffKV = kQ;
    static constexpr int kOffP = kOffKV + kNst * kStage;
    static constexpr int kBytes = kOffP + 4 * kP;   // P hi / lo, double buffered
};

// p as a hi + lo pair of 16-bit values (hi = round(p), lo = round(p - hi)),
// two columns at a time.
template <typename T> SDL_DEV void split_pair(float p0, float p1, uint32_t& hi, uint32_t& lo);
template <> SDL_DEV void split_pair<__nv_bfloat16>(float p0, float p1, uint32_t& hi, uint32_t& lo) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(p0, p1);
    const float2 hf = __bfloat1622float2(h);
    const __nv_bfloat162 l = __floats2bfloat162_rn(p0 - hf.x, p1 - hf.y);
    hi = *reinterpret_cast<const uint32_t*>(&h);
    lo = *reinterpret_cast<const uint32_t*>(&l);
}
template <> SDL_DEV void split_pair<__half>(float p0, float p1, uint32_t& hi, uint32_t& lo) {
    const __half2 h = __floats2half2_rn(p0, p1);
    const float2 hf = __half22float2(h);
    const __half2 l = __floats2half2_rn(p0 - hf.x, p1 - hf.y);
    hi = *reinterpret_cast<const uint32_t*>(&h);
    lo = *reinterpret_cast<const uint32_t*>(&l);
}

// The pair holding global tile `pos`: the last pair whose first tile is <= pos
// (empty pairs share their successor's first tile and are skipped this way).
SDL_DEV int sk_pair_of(const int* first, int npairs, int pos) {
    int lo = 0, hi = npairs;  // invariant: first[lo] <= pos < first[hi] (first[npairs] = total)
    while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (first[mid] <= pos) lo = mid; else hi = mid;
    }
    return lo;
}

// Rows of sequence b: position limit for query row j and whether it is valid.
SDL_DEV int sk_nvalid(const TcParams& p, int b) { return p.valid_rows ? min(p.valid_rows[b], p.chunk) : p.chunk; }

template <int HD, typename T>
__global__ void __launch_bounds__(kUThreads, 1)
attn_sk_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv, const TcParams p) {
    using L = USmem<HD>;
    constexpr int kUNst = L::kNst;
    constexpr int DO = L::DO;
    constexpr int SK = HD / 16;  // k-steps of the S product
    constexpr int OH = HD / 2;   // O columns per softmax thread
    constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
    constexpr uint32_t kIdescS = umma_idesc_f16(kURows, kUTok, kBf16, false);
    constexpr uint32_t kIdescO = umma_idesc_f16(kURows, HD, kBf16, true);
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    __shared__ uint64_t kv_full[kUNst], kv_empty[kUNst], s_full[2], s_free[2], p_full[2], p_free[2];
    __shared__ uint64_t q_full[2], q_free[2], o_free[2];
    __shared__ int s_first[kSkMaxPairs + 1];  // first global tile of each pair (prefix of tiles)
    __shared__ int s_start[kSkMaxSeqs], s_row[kSkMaxSeqs], s_nval[kSkMaxSeqs];  // per sequence
    __shared__ int s_slot[kSkMaxPairs];       // first partial slot of each pair
    __shared__ int s_red[32];
    __shared__ uint32_t s_tmem;
    __shared__ int s_abort_flag;
    volatile int* s_abort = &s_abort_flag;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int npairs = p.B * p.Hkv;
    const int G = gridDim.x, c = blockIdx.x;

    // --- per-sequence data, tile prefix over the pairs, tiles per CTA, slots.
    // Computed before griddepcontrol.wait, while the preceding kernel may
    // still run: no kernel of this library that lets its dependents start
    // early writes starts, valid_rows, rows or the block table.  The pair
    // table in the workspace, which the preceding split merge may still
    // read, is written only after the wait.
    for (int b = threadIdx.x; b < p.B; b += blockDim.x) {
        s_start[b] = p.starts[b];
        s_nval[b] = sk_nvalid(p, b);
        s_row[b] = p.dense ? 0 : p.rows[b];
    }
    __syncthreads();
    int total = 0;
    for (int base = 0; base < npairs; base += blockDim.x) {
        const int idx = base + threadIdx.x;
        int n = 0;
        if (idx < npairs) {
            const int b = idx / p.Hkv;
            const int lmax = s_start[b] + s_nval[b];
            n = lmax > 0 ? ((lmax + kPage - 1) / kPage + kUPages - 1) / kUPages : 0;
        }
        int tot;
        const int ex = block_exclusive_scan<int>(n, s_red, &tot);
        if (idx < npairs) s_first[idx] = total + ex;
        total += tot;
    }
    if (threadIdx.x == 0) s_first[npairs] = total;
    __syncthreads();
    const int tpc = (total + G - 1) / G;  // tiles per CTA
    int nslots = 0;
    for (int base = 0; base < npairs; base += blockDim.x) {
        const int idx = base + threadIdx.x;
        int cnt = 0;
        if (idx < npairs) {
            const int f = s_first[idx], n = s_first[idx + 1] - f;
            cnt = n > 0 ? (f + n - 1) / tpc - f / tpc + 1 : 0;
        }
        int tot;
        const int ex = block_exclusive_scan<int>(cnt, s_red, &tot);
        if (idx < npairs) s_slot[idx] = nslots + ex;
        nslots += tot;
    }
    __syncthreads();
    pdl_wait();
    if (c == 0) {
        for (int idx = threadIdx.x; idx < npairs; idx += blockDim.x) {
            const int f = s_first[idx], n = s_first[idx + 1] - f;
            const int cnt = n > 0 ? (f + n - 1) / tpc - f / tpc + 1 : 0;
            p.sk_table[idx] = make_int4(f, n, s_slot[idx], cnt);
        }
    }
    const int lo = c * tpc, hi = min(total, lo + tpc);
    if (lo >= hi) return;
    const int ntl = hi - lo;  // tiles of this CTA
    const int R = p.chunk * p.ratio;
    const int nsoft = (R + 15) / 16;
    // P as a hi + lo pair of 16-bit values (fp32 output keeps ~16 mantissa bits
    // of every weight); 16-bit outputs carry P rounded once, as their own
    // rounding already bounds the result to that precision.
    const bool p_split = p.out_dtype == SDL_F32;

    uint8_t* sQ = smem;
    uint8_t* sKV = smem + L::kOffKV;
    uint8_t* sP = smem + L::kOffP;
    const uint32_t aQ = smem_u32(sQ), aKV = smem_u32(sKV), aP = smem_u32(sP);

    if (threadIdx.x == 0) {
        *s_abort = 0;
        for (int i = 0; i < kUNst; ++i) {
            mbar_init(&kv_full[i], 1);
            mbar_init(&kv_empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&s_full[i], 1);
            mbar_init(&s_free[i], nsoft);
            mbar_init(&p_full[i], nsoft);
            mbar_init(&p_free[i], 1);
            mbar_init(&q_full[i], nsoft);
            mbar_init(&q_free[i], 1);
            mbar_init(&o_free[i], nsoft);
        }
        fence_mbar_init();
    }
    if (warp == kUMma) {
        tmem_alloc(&s_tmem, kUTmemCols);
        tmem_relinquish();
    }
    if (warp < 4) {
        // rows >= chunk*ratio stay zero in both Q buffers and all P matrices
        const int m = 16 * warp + (lane & 15), hq = lane >> 4;
        if (m >= R) {
#pragma unroll
            for (int cc = hq * (HD / 16); cc < (hq + 1) * (HD / 16); ++cc)
                *reinterpret_cast<uint4*>(sQ + (cc >> 3) * (kURows * 128) + m * 128 + (cc & 7) * 16) =
                    make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
            for (int mm = 0; mm < 4; ++mm)
#pragma unroll
                for (int cc = 4 * hq; cc < 4 * hq + 4; ++cc)
                    *reinterpret_cast<uint4*>(sP + mm * L::kP + m * 128 + (cc << 4)) = make_uint4(0u, 0u, 0u, 0u);
        }
        fence_proxy_async_smem();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_tmem;

    if (warp == kUProducer) {
        // ------------------------------------------------------- producer
        if (lane == 0) { prefetch_tmap(&tmk); prefetch_tmap(&tmv); }
        int issued = 0;
        bool stop = false;
        for (int i0 = 0; i0 < ntl && !stop; i0 += 32) {
            // lane l resolves tile i0 + l: its kv head and the first token of each page
            int tok[kUPages], head = 0;
#pragma unroll
            for (int u = 0; u < kUPages; ++u) tok[u] = 0;
            if (i0 + lane < ntl) {
                const int pos = lo + i0 + lane;
                const int idx = sk_pair_of(s_first, npairs, pos);
                const int b = idx / p.Hkv, tile = pos - s_first[idx];
                head = idx % p.Hkv;
                const int lmax = s_start[b] + s_nval[b];
                const int npg = (lmax + kPage - 1) / kPage;
                const int row = s_row[b];
#pragma unroll
                for (int u = 0; u < kUPages; ++u) {
                    int pg = tile * kUPages + u;
                    if (pg >= npg) pg = tile * kUPages;  // pad a short tile with a real page; masked later
                    if (p.dense) {
                        tok[u] = b * p.kv_len + pg * kPage;
                    } else {
                        int phys = pg < p.width ? p.table[(int64_t)row * p.width + pg] : -1;
                        if (phys < 0 || phys >= p.capacity) { sdl_raise(p.err, SDL_DEVERR_BAD_INDEX); phys = 0; }
                        tok[u] = (p.layer * p.capacity + phys) * kPage;
                    }
                }
            }
            const int cnt = min(32, ntl - i0);
            for (int k = 0; k < cnt; ++k) {
                const int i = i0 + k;
                const int st = i % kUNst;
                int t0[kUPages];
#pragma unroll
                for (int u = 0; u < kUPages; ++u) t0[u] = __shfl_sync(0xffffffffu, tok[u], k);
                const int gh = __shfl_sync(0xffffffffu, head, k);
                int ok = 1;
                if (i >= kUNst && lane == 0)
                    ok = mbar_wait_bounded(&kv_empty[st], ((i / kUNst) - 1) & 1, kWaitLimit) ? 1 : 0;
                ok = __shfl_sync(0xffffffffu, ok, 0);
                if (!ok || *s_abort) {
                    if (lane == 0 && !ok) { sdl_raise(p.err, SDL_DEVERR_TIMEOUT); *s_abort = 1; }
                    stop = true;
                    break;
                }
                // lane 0 posts the byte count, then one lane per 2 KB box issues it
                if (lane == 0) mbar_arrive_expect_tx(&kv_full[st], L::kStage);
                __syncwarp();
                if (lane < 2 * kUPages * DO) {
                    const int u = lane % kUPages, dd = (lane / kUPages) % DO, isv = lane / (kUPages * DO);
                    const int tu = u == 0 ? t0[0] : u == 1 ? t0[1] : u == 2 ? t0[2] : t0[3];
                    uint8_t* dst = sKV + st * L::kStage + (isv * DO + dd) * L::kHalf + u * kBoxBytes;
                    tma_load_4d(dst, isv ? &tmv : &tmk, &kv_full[st], 0, dd, gh, tu);
                }
                __syncwarp();
                issued = i + 1;
            }
        }
        // Never leave the CTA with bulk copies still landing in shared memory.
        if (lane == 0 && *s_abort) {
            for (int i = max(0, issued - kUNst); i < issued; ++i)
                (void)mbar_wait_bounded(&kv_full[i % kUNst], (i / kUNst) & 1, kWaitLimit);
        }
        pdl_launch_dependents();
    } else if (warp == kUMma) {
        // ------------------------------------------------------------ MMA
        if (lane == 0) {
            // Descriptors of the operand bases; an MMA adds its byte offset >> 4
            // to the start-address field (shared addresses stay below 2^18).
            const uint64_t dQ = umma_desc_sw128(aQ, 16, 1024);
            const uint64_t dK = umma_desc_sw128(aKV, 16, 1024);
            const uint64_t dP = umma_desc_sw128(aP, 16, 1024);
            const uint64_t dV = umma_desc_sw128(aKV + DO * L::kHalf, L::kHalf, 1024);
            int s_issued = 0, pv_issued = 0;
            bool ok = true;
            // Cursors (pair, segment ordinal) of the next S and the next PV.
            // The thread polls both and issues whichever is ready, so a PV
            // whose P is done never waits behind the next tile's K/V copy.
            int s_idx = sk_pair_of(s_first, npairs, lo), s_seg = 0;
            int v_idx = s_idx, v_seg = 0;
            uint32_t idle = 0;
            while (pv_issued < ntl) {
                if (*s_abort) { ok = false; break; }
                bool progress = false;
                if (pv_issued < s_issued) {
                    // ---- PV(i): O[64 x d] += P_hi V + P_lo V
                    const int i = pv_issued, pos = lo + i;
                    int vi = v_idx, vs = v_seg;
                    if (pos >= s_first[vi + 1]) { vi = sk_pair_of(s_first, npairs, pos); ++vs; }
                    const bool first = pos == max(lo, s_first[vi]);
                    const int pb = i & 1, st = i % kUNst;
                    const int ob = vs & 1;  // O buffer vs & 1 was last read by the epilogue of segment vs - 2
                    if (mbar_test_wait(&p_full[pb], (i >> 1) & 1) &&
                        (!first || vs < 2 || mbar_test_wait(&o_free[ob], ((vs - 2) >> 1) & 1))) {
                        v_idx = vi;
                        v_seg = vs;
                        tc_fence_after();
                        for (int h = 0; h < (p_split ? 2 : 1); ++h)
#pragma unroll
                            for (int k = 0; k < kUTok / 16; ++k) {
                                const uint32_t po = (2 * pb + h) * L::kP + k * 32;
                                const uint32_t vo = st * L::kStage + k * 2048;
                                umma_f16(tmem + kUOCol + ob * 128, dP + (po >> 4), dV + (vo >> 4), kIdescO,
                                         (!first || h > 0 || k > 0) ? 1u : 0u);
                            }
                        umma_commit(&p_free[pb]);
                        umma_commit(&kv_empty[st]);
                        pv_issued = i + 1;
                        progress = true;
                    }
                }
                if (s_issued < ntl) {
                    // ---- S(t) = Q K^T into TMEM buffer t & 1
                    const int t = s_issued, pos = lo + t;
                    int si = s_idx, ss = s_seg;
                    if (pos >= s_first[si + 1]) { si = sk_pair_of(s_first, npairs, pos); ++ss; }
                    const bool seg_first = pos == max(lo, s_first[si]);
                    const int st = t % kUNst, sb = t & 1;
                    if ((!seg_first || mbar_test_wait(&q_full[0], ss & 1)) &&
                        mbar_test_wait(&kv_full[st], (t / kUNst) & 1) &&
                        (t < 2 || mbar_test_wait(&s_free[sb], ((t - 2) >> 1) & 1))) {
                        s_idx = si;
                        s_seg = ss;
                        tc_fence_after();
#pragma unroll
                        for (int k = 0; k < SK; ++k) {
                            const uint32_t qo = (k >> 2) * (kURows * 128) + (k & 3) * 32;
                            const uint32_t ko = st * L::kStage + (k >> 2) * L::kHalf + (k & 3) * 32;
                            umma_f16(tmem + sb * kUTok, dQ + (qo >> 4), dK + (ko >> 4), kIdescS, k > 0 ? 1u : 0u);
                        }
                        umma_commit(&s_full[sb]);
                        // the segment's last S: the Q buffer may be refilled once it completes
                        if (pos == min(hi, s_first[si + 1]) - 1) umma_commit(&q_free[0]);
                        s_issued = t + 1;
                        progress = true;
                    }
                }
                if (progress) {
                    idle = 0;
                } else {
                    if (++idle > kPollLimit) { ok = false; break; }
                    __nanosleep(32);  // leave the issue slots to the softmax warp sharing this sub-partition
                }
            }
            if (!ok) {
                sdl_raise(p.err, SDL_DEVERR_TIMEOUT);
                *s_abort = 1;
            }
            // every issued MMA completes before TMEM is released
            if (s_issued > 0) (void)mbar_wait_bounded(&s_full[(s_issued - 1) & 1], ((s_issued - 1) >> 1) & 1, kWaitLimit);
            if (pv_issued > 0)
                (void)mbar_wait_bounded(&p_free[(pv_issued - 1) & 1], ((pv_issued - 1) >> 1) & 1, kWaitLimit);
        }
        __syncwarp();
        pdl_launch_dependents();
    } else if (warp < nsoft) {
        // ------------------------------------------------------- softmax
        const int hc = lane >> 4;               // column half of S (and of O)
        const int m = 16 * warp + (lane & 15);  // query row
        const int jr = m / p.ratio, hl = m % p.ratio;
        const uint32_t lane_base = (uint32_t)(32 * warp) << 16;
        bool ok = true;

        // Q rows of a segment's pair into the Q buffer (rows >= R stay zero):
        // 16-byte async copies now, published to the MMA thread later.
        auto issue_q = [&](int idx) {
            const int b = idx / p.Hkv, head = idx % p.Hkv;
            if (m < R) {
                const bool live = jr < s_nval[b];
                const T* qrow = reinterpret_cast<const T*>(p.q) + b * p.q_sb + jr * p.q_sj +
                                (head * p.ratio + hl) * p.q_sh;
#pragma unroll
                for (int cc = hc * (HD / 16); cc < (hc + 1) * (HD / 16); ++cc) {
                    uint8_t* dst = sQ + (cc >> 3) * (kURows * 128) + m * 128 + (((cc & 7) ^ (m & 7)) << 4);
                    if (live) cp_async16(dst, qrow + 8 * cc);
                    else *reinterpret_cast<uint4*>(dst) = make_uint4(0u, 0u, 0u, 0u);
                }
            }
        };
        auto publish_q = [&]() {
            cp_async_wait_all();
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(&q_full[0]);
        };

        int idx = sk_pair_of(s_first, npairs, lo), seg = 0;
        issue_q(idx);
        publish_q();
        int i = 0;
        while (i < ntl && ok) {
            // ---- one segment: tiles [seg_lo, seg_hi) of pair idx (global positions)
            const int seg_lo = max(lo, s_first[idx]), seg_hi = min(hi, s_first[idx + 1]);
            const int b = idx / p.Hkv, head = idx % p.Hkv;
            const int start = s_start[b], nvalid = s_nval[b];
            const int ob = seg & 1;  // O buffer of this segment
            const bool live = m < R && jr < nvalid;
            const int npg = (start + nvalid + kPage - 1) / kPage;
            const int lim = live ? start + jr + 1 : 0;  // the row attends positions < lim
            const int lim_eff = min(lim, npg * kPage);
            const int tile0 = seg_lo - s_first[idx];    // first tile of the segment within the pair
            // the next segment's Q refills the buffer once this segment's last S is done
            const bool stage_next = seg_hi < hi;
            float m_run = -INFINITY, l_run = 0.f;
            for (int pos = seg_lo; pos < seg_hi; ++pos, ++i) {
                const int sb = i & 1, pb = i & 1;
                ok = __all_sync(0xffffffffu, mbar_wait_bounded(&s_full[sb], (i >> 1) & 1, kWaitLimit));
                if (!ok || *s_abort) { ok = false; break; }
                tc_fence_after();
                float sv[32];
                __syncwarp();
                tmem_ld16x2<32>(tmem + lane_base + sb * kUTok, reinterpret_cast<uint32_t*>(sv));
                tmem_wait_ld();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&s_free[sb]);
                if (stage_next && pos == seg_hi - 1) {
                    // S of the segment's last tile is done, and with it every read of Q
                    ok = __all_sync(0xffffffffu, mbar_wait_bounded(&q_free[0], seg & 1, kWaitLimit));
                    if (!ok) break;
                    issue_q(sk_pair_of(s_first, npairs, seg_hi));
                }

                // raw scores; positions at or past the row's limit are masked
                const int c0 = (tile0 + pos - seg_lo) * kUTok + 32 * hc;
                if (c0 + 32 > lim_eff) {
#pragma unroll
                    for (int cc = 0; cc < 32; ++cc) sv[cc] = c0 + cc < lim_eff ? sv[cc] : -INFINITY;
                }
                float tmax = sv[0];
#pragma unroll
                for (int cc = 1; cc < 32; ++cc) tmax = fmaxf(tmax, sv[cc]);
                tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 16));
                const float m_new = fmaxf(m_run, tmax * p.scale_log2);
                const bool need = m_new > m_run + 8.f;
                if (pos > seg_lo && __any_sync(0xffffffffu, need)) {
                    // O is rescaled in place once PV(i-1) has landed
                    ok = __all_sync(0xffffffffu,
                                    mbar_wait_bounded(&p_free[(i - 1) & 1], ((i - 1) >> 1) & 1, kWaitLimit));
                    if (!ok) break;
                    tc_fence_after();
                    const float alpha = need ? exp2f(m_run - m_new) : 1.f;
#pragma unroll
                    for (int o0 = 0; o0 < OH; o0 += 32) {
                        uint32_t o[32];
                        __syncwarp();
                        tmem_ld16x2<OH>(tmem + lane_base + kUOCol + ob * 128 + o0, o);
                        tmem_wait_ld();
#pragma unroll
                        for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
                        tmem_st16x2<OH>(tmem + lane_base + kUOCol + ob * 128 + o0, o);
                    }
                    tmem_wait_st();
                    l_run *= alpha;
                }
                if (need) m_run = m_new;
                const float muse = m_run == -INFINITY ? 0.f : m_run;
                if (i >= 2) {
                    ok = __all_sync(0xffffffffu, mbar_wait_bounded(&p_free[pb], ((i - 2) >> 1) & 1, kWaitLimit));
                    if (!ok) break;
                }
                if (m < R) {
                    float lsum = 0.f;
                    uint8_t* ph = sP + (2 * pb) * L::kP + m * 128;
                    uint8_t* pl = sP + (2 * pb + 1) * L::kP + m * 128;
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        uint32_t hw[4], lw[4];
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const float p0 = ex2_approx(fmaf(sv[8 * k + 2 * e], p.scale_log2, -muse));
                            const float p1 = ex2_approx(fmaf(sv[8 * k + 2 * e + 1], p.scale_log2, -muse));
                            lsum += p0 + p1;
                            if (p_split) split_pair<T>(p0, p1, hw[e], lw[e]);
                            else hw[e] = pack2<T>(p0, p1);
                        }
                        const int sw = ((4 * hc + k) ^ (m & 7)) << 4;
                        *reinterpret_cast<uint4*>(ph + sw) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
                        if (p_split) *reinterpret_cast<uint4*>(pl + sw) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
                    }
                    l_run += lsum;
                }
                fence_proxy_async_smem();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&p_full[pb]);
                if (stage_next && pos == seg_hi - 1) publish_q();  // the copies overlapped this tile's softmax
            }
            if (!ok) break;
            // ---- segment epilogue
            const float l_tot = l_run + __shfl_xor_sync(0xffffffffu, l_run, 16);
            const int last = i - 1;
            ok = __all_sync(0xffffffffu, mbar_wait_bounded(&p_free[last & 1], (last >> 1) & 1, kWaitLimit));
            if (!ok) break;
            tc_fence_after();
            const int f = s_first[idx], n = s_first[idx + 1] - f;
            const bool whole = (f / tpc == c) && ((f + n - 1) / tpc == c);  // this CTA owns the pair
            const int slot = s_slot[idx] + (c - f / tpc);
            const int h = head * p.ratio + hl;
            const int64_t part = (int64_t)slot * R + m;
            const float inv = 1.f / l_tot;
#pragma unroll
            for (int o0 = 0; o0 < OH; o0 += 32) {
                uint32_t o[32];
                __syncwarp();  // TMEM loads are warp-collective: converge first
                tmem_ld16x2<OH>(tmem + lane_base + kUOCol + ob * 128 + o0, o);
                tmem_wait_ld();
                const int d0 = hc * OH + o0;
                if (live && whole) {
                    const int64_t ob = b * p.o_sb + jr * p.o_sj + h * p.o_sh + d0;
#pragma unroll
                    for (int e = 0; e < 32; ++e) store_from_f32(p.out, ob + e, p.out_dtype, __uint_as_float(o[e]) * inv);
                } else if (m < R && !whole) {
                    float4* dst = reinterpret_cast<float4*>(p.o_part + part * HD + d0);
#pragma unroll
                    for (int e = 0; e < 8; ++e)
                        dst[e] = make_float4(__uint_as_float(o[4 * e]), __uint_as_float(o[4 * e + 1]),
                                             __uint_as_float(o[4 * e + 2]), __uint_as_float(o[4 * e + 3]));
                }
            }
            if (m < R && !whole && hc == 0) {
                p.ml_part[part * 2] = m_run;
                p.ml_part[part * 2 + 1] = l_tot;
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&o_free[ob]);
            // next segment
            if (seg_hi < hi) {
                idx = sk_pair_of(s_first, npairs, seg_hi);
                ++seg;
            }
        }
        pdl_launch_dependents();
        if (!ok && lane == 0) {
            sdl_raise(p.err, SDL_DEVERR_TIMEOUT);
            *s_abort = 1;
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == kUMma) tmem_dealloc(tmem, kUTmemCols);
}

// Merge the partials of pairs split across CTAs: one warp per (pair, query
// row), each lane owning 4 head dims.  Up to kCombineOneRound slots take one
// round of loads (every slot's m, l and this lane's dims of its row at once);
// more take a reduction of the slot maxima and sums across lanes, then the
// rows slot by slot.  A slot whose tiles lie past the row's key limit holds
// m = -inf and weighs 0.
__global__ void __launch_bounds__(128) attn_sk_combine_kernel(TcParams p, int hd) {
    pdl_wait();
    pdl_launch_dependents();  // the next launch may become resident; it waits for this grid to finish
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int R = p.chunk * p.ratio;
    const int wr = blockIdx.x * 4 + warp;
    if (wr >= p.B * p.Hkv * R) return;
    const int idx = wr / R, m = wr % R;
    const int4 t = p.sk_table[idx];
    const int cnt = t.w;
    if (cnt <= 1) return;
    const int b = idx / p.Hkv, head = idx % p.Hkv;
    const int j = m / p.ratio, h = head * p.ratio + m % p.ratio;
    const int nvalid = p.valid_rows ? min(p.valid_rows[b], p.chunk) : p.chunk;
    if (j >= nvalid) return;
    const int64_t base = (int64_t)t.z * R + m;  // partial of slot t.z, row m
    if (cnt <= kCombineOneRound && hd <= 128) {
        const int d0 = lane * 4;
        const bool mine = d0 < hd;
        float2 ml[kCombineOneRound];
        float4 o[kCombineOneRound];
#pragma unroll
        for (int s = 0; s < kCombineOneRound; ++s) {
            ml[s] = make_float2(-INFINITY, 0.f);
            o[s] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (s < cnt) {
                const int64_t row = base + (int64_t)s * R;
                ml[s] = *reinterpret_cast<const float2*>(p.ml_part + row * 2);
                if (mine) o[s] = *reinterpret_cast<const float4*>(p.o_part + row * hd + d0);
            }
        }
        float M = -INFINITY;
#pragma unroll
        for (int s = 0; s < kCombineOneRound; ++s) M = fmaxf(M, ml[s].x);
        float den = 0.f;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int s = 0; s < kCombineOneRound; ++s) {
            const float w = ex2_approx(ml[s].x - M);  // 0 for -inf maxima and the padding slots
            den = fmaf(w, ml[s].y, den);
            acc.x = fmaf(w, o[s].x, acc.x);
            acc.y = fmaf(w, o[s].y, acc.y);
            acc.z = fmaf(w, o[s].z, acc.z);
            acc.w = fmaf(w, o[s].w, acc.w);
        }
        if (mine) {
            const float inv = 1.f / den;
            const int64_t ob = b * p.o_sb + j * p.o_sj + h * p.o_sh + d0;
            store_from_f32(p.out, ob, p.out_dtype, acc.x * inv);
            store_from_f32(p.out, ob + 1, p.out_dtype, acc.y * inv);
            store_from_f32(p.out, ob + 2, p.out_dtype, acc.z * inv);
            store_from_f32(p.out, ob + 3, p.out_dtype, acc.w * inv);
        }
        return;
    }
    float M = -INFINITY;
    for (int s = lane; s < cnt; s += 32) M = fmaxf(M, p.ml_part[(base + (int64_t)s * R) * 2]);
    M = warp_max(M);
    float den = 0.f;
    for (int s = lane; s < cnt; s += 32) {
        const float* ml = p.ml_part + (base + (int64_t)s * R) * 2;
        den += ml[0] == -INFINITY ? 0.f : exp2f(ml[0] - M) * ml[1];
    }
    den = warp_sum(den);
    const float inv = 1.f / den;
    const int64_t ob = b * p.o_sb + j * p.o_sj + h * p.o_sh;
    for (int d0 = lane * 4; d0 < hd; d0 += 128) {
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int s = 0; s < cnt; ++s) {
            const int64_t row = base + (int64_t)s * R;
            const float mv = p.ml_part[row * 2];
            const float wt = mv == -INFINITY ? 0.f : exp2f(mv - M);
            const float4 o = *reinterpret_cast<const float4*>(p.o_part + row * hd + d0);
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

// ------------------------------------------------------ positional append
// New K/V rows [B*chunk][Hkv*d] stored at positions starts[b] + j (j below the
// valid rows) of each sequence's pages: the append half of a fused call on
// the paths that do not write inside the attention kernel.  One warp per row.
__global__ void __launch_bounds__(128) kv_append_pos_kernel(TcParams p, int row_bytes, int bs) {
    const int r = blockIdx.x * 4 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (r >= p.B * p.chunk) return;
    const int b = r / p.chunk, j = r % p.chunk;
    const int nvalid = p.valid_rows ? min(p.valid_rows[b], p.chunk) : p.chunk;
    if (j >= nvalid) return;
    const int pos = p.starts[b] + j;
    if (pos < 0) return;
    const int pg = pos / bs;
    const int row = p.rows[b];
    const int phys = pg < p.width ? p.table[(int64_t)row * p.width + pg] : -1;
    if (phys < 0 || phys >= p.capacity) {
        if (lane == 0) sdl_raise(p.err, SDL_DEVERR_BAD_INDEX);
        return;
    }
    const int64_t dst = ((int64_t)(p.layer * p.capacity + phys) * bs + pos % bs) * row_bytes;
    const int64_t src = (int64_t)r * p.new_stride;
    for (int o = lane * 4; o < row_bytes; o += 128) {
        *reinterpret_cast<uint32_t*>(p.k_pool + dst + o) = *reinterpret_cast<const uint32_t*>(p.k_new + src + o);
        *reinterpret_cast<uint32_t*>(p.v_pool + dst + o) = *reinterpret_cast<const uint32_t*>(p.v_new + src + o);
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
    int ring_bytes = 0;    // shared bytes before the mbarriers (ring, or cluster partials when larger)
    bool cluster = false;  // splits of a row form one cluster and merge on chip
    bool rows = false;     // rows-on-M mma.sync kernel (ncoltiles = row tiles, wpg = consumer warps)
    bool umma = false;     // tcgen05 verify kernel
    bool direct = false;   // register-direct decode kernel (one CTA per split, kv head and sequence)
    int stages = 0;        // rows-on-M kernel: ring depth
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

// The persistent tcgen05 kernel takes row blocks of up to 64 query rows per
// kv head and up to 512 (sequence, kv head) pairs.  It runs when asked for
// (use_umma = 1); the automatic plan keeps the mma.sync kernel.
bool umma_applicable(const sdl_attn_args* a) {
    if (a->use_umma < 0 || !tc_applicable(a)) return false;
    // Q rows are staged with 16-byte async copies
    if (((a->q_sb | a->q_sj | a->q_sh) & 7) || reinterpret_cast<uintptr_t>(a->q) % 16) return false;
    const int rows = a->chunk * (a->Hq / a->Hkv);
    if (rows > kURows || (long)a->B * a->Hkv > kSkMaxPairs) return false;
    if (a->use_umma > 0) return true;
    if (a->key_count < 0) return false;  // ragged rows of unknown lengths: the mma.sync plans
    // Automatic choice: the mma.sync kernels spend many issue slots per
    // page, so large blocks over long contexts are instruction bound there;
    // the tcgen05 kernel issues the products from one thread.  Measured on
    // B200: 56 rows per kv head over 8k-32k keys (C5 verify) 87.7 us against
    // 100 (rows on M) / 116 (keys on M); 30 rows over 8k-32k keys 93.7
    // against 75.1 (keys on M); 30 rows over mostly short rows with one of
    // 4200 keys 42.0 against 25.8 (rows on M).  The mean span decides (the
    // key count when given), not the longest row.
    const long mean_keys = a->key_count > 0 ? (long)(a->key_count / std::max(1, a->B)) : (long)a->max_limit;
    return rows >= kUmmaAutoMinRows && mean_keys >= kUmmaAutoMinKeys;
}

// Workspace of the persistent kernel: the per-pair table, then fp32 partials
// for at most (grid + pairs) slots of chunk*ratio rows.
size_t sk_header_bytes(int npairs) { return ((size_t)npairs * sizeof(int4) + 255) & ~size_t(255); }

Plan make_umma_plan(const sdl_attn_args* a) {
    Plan pl;
    pl.tc = true;
    pl.umma = true;
    pl.smem = (a->head_dim == 128 ? USmem<128>::kBytes : USmem<64>::kBytes) + 1024;
    const int max_pages = std::max(1, (a->max_limit + kPage - 1) / kPage);
    const long tiles_upper = (long)a->B * a->Hkv * ((max_pages + kUPages - 1) / kUPages);
    pl.nsplit = (int)std::max(1L, std::min<long>(sm_count(), tiles_upper));  // persistent grid
    pl.pps = kUPages;
    const int npairs = a->B * a->Hkv;
    const int rows = a->chunk * (a->Hq / a->Hkv);
    pl.ws_bytes = sk_header_bytes(npairs) + (size_t)(pl.nsplit + npairs) * rows * (a->head_dim + 2) * sizeof(float);
    return pl;
}

// Per-instantiation kernel attributes: the dynamic shared-memory ceiling
// (raised monotonically), all of the unified L1/shared array as shared memory
// (the ring buffers, not L1, decide how many CTAs an SM holds) and clusters
// of up to kMaxClusterSplits CTAs.
template <int HD, int NTG, typename T>
int tc_configure(size_t smem) {
    static std::mutex mu;
    static size_t configured = 0;
    std::lock_guard<std::mutex> lock(mu);
    if (smem <= configured) return SDL_OK;
    auto kern = attn_tc_kernel<HD, NTG, T>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, (int)cudaSharedmemCarveoutMaxShared);
    if (e == cudaSuccess) e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) return sdl::fail(SDL_ERR_CUDA, cudaGetErrorString(e));
    configured = smem;
    return SDL_OK;
}

// Whether clusters of `nsplit` CTAs of this kernel can be resident at all
// (cached per shape; any failure answers no and the plan falls back to the
// workspace merge).
template <int HD, int NTG, typename T>
bool tc_cluster_fits_inst(int nsplit, size_t smem, int threads) {
    static std::mutex mu;
    static std::vector<std::pair<uint64_t, bool>> cache;
    const uint64_t key = ((uint64_t)nsplit << 48) | ((uint64_t)threads << 32) | (uint64_t)smem;
    {
        std::lock_guard<std::mutex> lock(mu);
        for (const auto& kv : cache)
            if (kv.first == key) return kv.second;
    }
    bool ok = false;
    if (tc_configure<HD, NTG, T>(smem) == SDL_OK) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(nsplit, 1, 1);
        cfg.blockDim = dim3(threads);
        cfg.dynamicSmemBytes = smem;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = nsplit;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        int n = 0;
        ok = cudaOccupancyMaxActiveClusters(&n, attn_tc_kernel<HD, NTG, T>, &cfg) == cudaSuccess && n > 0;
        (void)cudaGetLastError();  // a refused query leaves no sticky error
    }
    std::lock_guard<std::mutex> lock(mu);
    cache.emplace_back(key, ok);
    return ok;
}

bool tc_cluster_fits(int hd, int ntg, int dtype, int nsplit, size_t smem, int threads) {
    if (dtype == SDL_BF16) {
        if (hd == 64) return ntg == 2 ? tc_cluster_fits_inst<64, 2, __nv_bfloat16>(nsplit, smem, threads)
                                      : tc_cluster_fits_inst<64, 1, __nv_bfloat16>(nsplit, smem, threads);
        return ntg == 2 ? tc_cluster_fits_inst<128, 2, __nv_bfloat16>(nsplit, smem, threads)
                        : tc_cluster_fits_inst<128, 1, __nv_bfloat16>(nsplit, smem, threads);
    }
    if (hd == 64) return ntg == 2 ? tc_cluster_fits_inst<64, 2, __half>(nsplit, smem, threads)
                                  : tc_cluster_fits_inst<64, 1, __half>(nsplit, smem, threads);
    return ntg == 2 ? tc_cluster_fits_inst<128, 2, __half>(nsplit, smem, threads)
                    : tc_cluster_fits_inst<128, 1, __half>(nsplit, smem, threads);
}

// Resident CTAs per SM of one instantiation at this shared-memory size and
// block (cached per shape; 0 when the query fails).
template <int HD, int NTG, typename T>
int tc_occupancy_inst(size_t smem, int threads) {
    static std::mutex mu;
    static std::vector<std::pair<uint64_t, int>> cache;
    const uint64_t key = ((uint64_t)threads << 32) | (uint64_t)smem;
    {
        std::lock_guard<std::mutex> lock(mu);
        for (const auto& kv : cache)
            if (kv.first == key) return kv.second;
    }
    int n = 0;
    if (tc_configure<HD, NTG, T>(smem) != SDL_OK ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, attn_tc_kernel<HD, NTG, T>, threads, smem) != cudaSuccess) {
        (void)cudaGetLastError();  // a refused query leaves no sticky error
        return 0;
    }
    std::lock_guard<std::mutex> lock(mu);
    cache.emplace_back(key, n);
    return n;
}

int tc_occupancy(int hd, int ntg, int dtype, size_t smem, int threads) {
    if (dtype == SDL_BF16) {
        if (hd == 64) return ntg == 2 ? tc_occupancy_inst<64, 2, __nv_bfloat16>(smem, threads)
                                      : tc_occupancy_inst<64, 1, __nv_bfloat16>(smem, threads);
        return ntg == 2 ? tc_occupancy_inst<128, 2, __nv_bfloat16>(smem, threads)
                        : tc_occupancy_inst<128, 1, __nv_bfloat16>(smem, threads);
    }
    if (hd == 64) return ntg == 2 ? tc_occupancy_inst<64, 2, __half>(smem, threads)
                                  : tc_occupancy_inst<64, 1, __half>(smem, threads);
    return ntg == 2 ? tc_occupancy_inst<128, 2, __half>(smem, threads)
                    : tc_occupancy_inst<128, 1, __half>(smem, threads);
}

constexpr int kMinSplitPages = 4;  // fewest pages per split-K CTA the automatic plan chooses
// Fill of the resident CTA slots the key-count plan aims at, measured on
// B200 over split sizes.  Decode (one query row per sequence; 64 rows
// U[512,4096], 144 rows U[200,1500], 16 rows U[8k,32k]) is bandwidth bound
// and fastest at 86-90 % (fewer, equal CTAs per SM); verify blocks (6-7 rows
// per sequence) are issue bound and fastest at 95-97 % (more resident warps).
// Fuller grids spill CTAs into a second wave.
constexpr double kOneWaveFillDecode = 0.89;
constexpr double kOneWaveFillBlock = 0.96;
// Automatic plans: query rows per kv head from which the rows-on-M kernel
// runs.  Measured on B200: it wins for head_dim 64 verify blocks (42 rows:
// 15.1 against 18.5 us), 56-row verify (100 against 116 us) and prefill;
// 36-row head_dim-128 verify is latency bound in both and the keys-on-M
// kernel, with more warps per SM, is 3 % faster there (32 rows of 256-2048
// keys).  Over short rows the balance turns: 30-row blocks of 64 sequences
// with a mean of ~700 keys take 24-26 us on rows on M against 32-33 us on
// keys on M, so head_dim-128 blocks of 24+ rows take rows on M when the key
// count puts the mean span below kRowsShortKeys.
constexpr int kRowsMinRows64 = 16;
constexpr int kRowsMinRows128 = 48;
constexpr int kRowsMinRows128Short = 24;
constexpr int kRowsShortKeys = 1024;

template <int HD, typename T>
int rows_configure(size_t smem) {
    static std::mutex mu;
    static size_t configured = 0;
    std::lock_guard<std::mutex> lock(mu);
    if (smem <= configured) return SDL_OK;
    auto kern = attn_rows_kernel<HD, T>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, (int)cudaSharedmemCarveoutMaxShared);
    if (e != cudaSuccess) return sdl::fail(SDL_ERR_CUDA, cudaGetErrorString(e));
    configured = smem;
    return SDL_OK;
}

template <int HD, typename T>
int rows_occupancy_inst(size_t smem, int threads) {
    static std::mutex mu;
    static std::vector<std::pair<uint64_t, int>> cache;
    const uint64_t key = ((uint64_t)threads << 32) | (uint64_t)smem;
    {
        std::lock_guard<std::mutex> lock(mu);
        for (const auto& kv : cache)
            if (kv.first == key) return kv.second;
    }
    int n = 0;
    if (rows_configure<HD, T>(smem) != SDL_OK ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, attn_rows_kernel<HD, T>, threads, smem) != cudaSuccess) {
        (void)cudaGetLastError();
        return 0;
    }
    std::lock_guard<std::mutex> lock(mu);
    cache.emplace_back(key, n);
    return n;
}

int rows_occupancy(int hd, int dtype, size_t smem, int threads) {
    if (dtype == SDL_BF16)
        return hd == 64 ? rows_occupancy_inst<64, __nv_bfloat16>(smem, threads)
                        : rows_occupancy_inst<128, __nv_bfloat16>(smem, threads);
    return hd == 64 ? rows_occupancy_inst<64, __half>(smem, threads) : rows_occupancy_inst<128, __half>(smem, threads);
}

// Pages per split-K CTA: without a key count, enough splits for ~4 CTAs per
// SM if every row spanned max_limit; with one, the fewest pages per split
// whose grid fills about kOneWaveFill* of the resident CTA slots (`occ` per
// SM).  Each work item holds about key_count / B keys and leaves on average
// half a split of remainder; a second wave for a few CTAs costs more than
// the per-SM balance smaller splits buy.
//
// key_count < 0 declares ragged rows of unknown lengths: a plan captured in
// a CUDA graph and replayed over other batches, of which only the grid's
// bounds (B, max_limit) are known.  A one-wave plan sized for max_limit
// leaves the longest rows of a skewed batch in one CTA each, and those
// CTAs set the launch's duration; tiny splits instead fill the grid with
// CTAs past short rows' ends and multiply the merge's partials.  So a
// split holds max(n/16, max_pages/16) pages for decode and max(n/16,
// max_pages/32) for blocks (n = the unsplit CTAs), within 8..64.  Measured
// on B200 over C4-shaped batches (contexts floor(lognormal(6, 0.8)) +
// U[0, 512) tokens) at the C4 pools' 4656-key span, fixed pages per split:
//   decode (14 q / 2 kv heads, d 64), pages 4 / 8 / 12 / 20 / 40:
//     16 seqs 9.7 / 8.0 / 8.5 / 9.4 / 12.6 us; 64 seqs 26.5 / 19.3 / 17.0 /
//     13.8 / 18.4; 256 seqs 48.7 / 34.6 / 31.2 / 28.9 / 35.0
//   5-row verify (12 q / 2 kv heads, d 128, rows on M):
//     16 seqs 15.5 / 13.9 / 15.7 / 20.6 / 30.6; 64 seqs 51.2 / 36.6 /
//     33.4 / 29.7 / 40.0; 256 seqs 175 / 114 / 94 / 82 / 79
// and, with the grid for an 8192-key span, verify at 358 / 512 / 1024
// sequences 110 / 144 / 266 us at 32 pages and 108 / 135 / 239 at 64,
// against 145 / 155 / 240 for the exact-count plan and 214 / 215 / 298 for
// a one-wave plan at 55 % of the span.
constexpr int kRaggedSplitDiv = 16;
// The register-direct kernel's splits grow with the grid at twice that rate
// (max(n/8, max_pages/16) pages; n = sequences x kv heads): measured on B200
// over the same C4-shaped draft batches, span bucket 2048 / 4656 keys, pages
// per split 8 / 12 / 16 / 24: 64 seqs 15.0 / 11.8 / 12.1 / 14.1 and 19.0 /
// 16.1 / 14.3 / 14.6 us; 96 seqs 19.1 / 17.8 / 17.2 / 15.1 and 25.3 / 21.5 /
// 21.7 / 17.2; at 8-48 seqs 8-12 pages (span 2048) and 12-19 (span 4656).
constexpr int kRaggedSplitDivDirect = 8;
constexpr int kRaggedMinSplitPages = 8;
constexpr int kRaggedBlockChunk = 32;  // positions per row from which a block is prefill-sized
constexpr int kRaggedMaxSplitPages = 64;
int split_pages(const sdl_attn_args* a, long base_ctas, int max_pages, int occ, int ragged_div = kRaggedSplitDiv) {
    if (a->pages_per_split > 0) return a->pages_per_split;
    if (a->key_count < 0) {
        const long span_div = a->chunk > 1 ? 32 : 16;
        long pps = std::max<long>(base_ctas / ragged_div, (max_pages + span_div - 1) / span_div);
        pps = std::min<long>(kRaggedMaxSplitPages, std::max<long>(kRaggedMinSplitPages, pps));
        if (a->chunk >= kRaggedBlockChunk) {
            // prefill-sized blocks: a split's fp32 partials (chunk x Hq rows)
            // outweigh the pages it saves, so rows split only as far as it
            // takes to give every SM a CTA.  (Splitting long rows at 64
            // pages as well measured no faster: a 2800-token prompt's
            // chunks cost 137 us per draft layer either way, plus 34 us of
            // merge -- the launch is bound by its quadratic MMA work, not by
            // its longest CTA.)
            const long want = (sm_count() + base_ctas - 1) / base_ctas;
            pps = std::max<long>(pps, (max_pages + want - 1) / want);
        }
        return (int)std::min<long>(pps, max_pages);
    }
    const long target = (long)sm_count() * 4;
    const int nsplit_target = (int)std::max(1L, (target + base_ctas - 1) / base_ctas);
    int pps = std::max(kMinSplitPages, (max_pages + nsplit_target - 1) / nsplit_target);
    if (a->key_count > 0 && occ > 0) {
        const double slots = (a->chunk == 1 ? kOneWaveFillDecode : kOneWaveFillBlock) * sm_count() * occ;
        const double row_pages = (double)a->key_count / ((double)a->B * kPage) + 0.5;
        int p2 = kMinSplitPages;
        while (p2 < max_pages && (double)base_ctas * (row_pages / p2 + 0.5) > slots) ++p2;
        pps = std::min(p2, max_pages);
    }
    return pps;
}

// Splits covering max_limit and their workspace; without enough caller
// workspace the split doubles until the partials fit.
void finish_split_plan(const sdl_attn_args* a, Plan& pl, int pps, int max_pages, int align) {
    for (;;) {
        pps = (pps + align - 1) / align * align;
        pl.pps = pps;
        pl.nsplit = (max_pages + pps - 1) / pps;
        pl.ws_bytes = pl.nsplit > 1 ? (size_t)a->B * pl.nsplit * a->chunk * a->Hq * (a->head_dim + 2) * sizeof(float) : 0;
        if (a->pages_per_split > 0 || pl.ws_bytes <= a->workspace_bytes || pl.nsplit == 1 || !a->workspace) break;
        pps *= 2;
    }
}

bool rows_applicable(const sdl_attn_args* a) {
    if (a->mma_layout == 1 || a->cluster_merge || !tc_applicable(a)) return false;
    if (a->mma_layout == 2) return true;
    const int rows = a->chunk * (a->Hq / a->Hkv);
    if (rows >= (a->head_dim == 64 ? kRowsMinRows64 : kRowsMinRows128)) return true;
    // ragged rows of unknown lengths (key_count < 0) split at most
    // kRaggedMaxSplitPages pages per CTA, where rows on M measured ahead
    // (C4 verify, 30 rows: 110 against 131 us at 358 sequences)
    return a->head_dim == 128 && rows >= kRowsMinRows128Short &&
           (a->key_count < 0 || (a->key_count > 0 && a->key_count < (int64_t)kRowsShortKeys * a->B));
}

Plan make_rows_plan(const sdl_attn_args* a) {
    Plan pl;
    pl.tc = true;
    pl.rows = true;
    const int R = a->chunk * (a->Hq / a->Hkv);
    pl.ncoltiles = (R + kRowTile - 1) / kRowTile;
    pl.wpg = (std::min(R, kRowTile) + 15) / 16;
    pl.g_cta = 1;
    pl.kvgroups = a->Hkv;
    pl.stage_bytes = a->head_dim == 128 ? rows_stage_bytes<128>() : rows_stage_bytes<64>();
    pl.stages = kRowStages;
    pl.ring_bytes = pl.stages * pl.stage_bytes;
    pl.smem = (size_t)pl.ring_bytes + 1024 + 2 * pl.stages * sizeof(uint64_t);
    const int max_pages = std::max(1, (a->max_limit + kPage - 1) / kPage);
    const long base_ctas = (long)a->B * pl.ncoltiles * pl.kvgroups;
    const int occ = a->key_count > 0 ? rows_occupancy(a->head_dim, a->dtype, pl.smem, (pl.wpg + 1) * 32) : 0;
    finish_split_plan(a, pl, split_pages(a, base_ctas, max_pages, occ), max_pages, kTilePages);
    return pl;
}

template <int HD, typename T>
int direct_occupancy_inst() {
    static int n = -1;
    static std::mutex mu;
    std::lock_guard<std::mutex> lock(mu);
    if (n < 0) {
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, attn_direct_kernel<HD, T>, kDirWarps * 32, 0) !=
            cudaSuccess) {
            (void)cudaGetLastError();
            return 0;  // not cached: a later call asks again
        }
    }
    return n;
}

int direct_occupancy(int hd, int dtype) {
    if (dtype == SDL_BF16)
        return hd == 64 ? direct_occupancy_inst<64, __nv_bfloat16>() : direct_occupancy_inst<128, __nv_bfloat16>();
    return hd == 64 ? direct_occupancy_inst<64, __half>() : direct_occupancy_inst<128, __half>();
}

// The register-direct kernel covers blocks of at most kDirCols query columns
// per kv head over 16-byte aligned K/V.  It runs when asked for
// (mma_layout = 3) and, automatically, for head_dim-64 decode over short
// rows (a key count with a mean span of at most kDirAutoMaxKeys), where it
// measured faster on B200 (0.5B-shaped draft, 64 rows of 200-1500 keys:
// 11.4-11.9 against 13.0 us).  Over 1000-3000 keys the TMA kernel is ahead
// (18.5 against 21.1 us), and at head_dim 128 the TMA ring keeps more bytes
// in flight per SM than the registers can (C2 decode 30.1 against 33.4 us).
constexpr int kDirAutoMaxKeys = 1280;
// ... except for mid-sized batches of such rows: 0.5B-shaped draft decode
// over C4 contexts (mean ~720 keys) measured 29.7 against 35.5 us at 256
// sequences and 48.7 against 77.4 us at 512 for the TMA kernel, while the
// register-direct kernel stays ahead at 64 (12.3 against 14.3 us) and at
// 1024 sequences (111 against 131 us).  Between these key counts the TMA
// kernel runs.
constexpr int64_t kDirMidKeysLo = 160 * 1024;
constexpr int64_t kDirMidKeysHi = 560 * 1024;
// Ragged rows of unknown lengths (key_count < 0, a captured forward): the
// register-direct kernel for head_dim-64 decode of up to kDirRaggedMaxRows
// sequences, where it skips the TMA ring's ramp.  0.5B-shaped draft decode
// over C4-shaped batches (contexts floor(lognormal(6, 0.8)) + U[0, 512)
// tokens, span buckets up to 4656 keys), graphs of 8 layers, measured on
// B200 against the keys-on-M TMA kernel, both with their ragged split rules
// (span bucket 4656 keys): 8 / 16 / 32 / 64 / 96 / 112 / 128 sequences
// 9.5 / 10.0 / 12.8 / 13.7 / 17.1 / 17.7 / 19.6 us against 16.4 / 15.9 /
// 18.5 / 18.4 / 19.8 / 20.1 / 20.3; at 160 they tie (22.1 / 21.8), and
// from 192 the TMA kernel is ahead (23.2 against 26.4; 358: 40.6 / 43.4).
constexpr int kDirRaggedMaxRows = 128;
bool direct_applicable(const sdl_attn_args* a) {
    if (a->mma_layout == 1 || a->mma_layout == 2 || a->cluster_merge || !tc_applicable(a)) return false;
    if (a->chunk * (a->Hq / a->Hkv) > kDirCols) return false;
    const void* k = a->k_pool ? a->k_pool : a->k_dense;
    const void* v = a->k_pool ? a->v_pool : a->v_dense;
    if (reinterpret_cast<uintptr_t>(k) % 16 || reinterpret_cast<uintptr_t>(v) % 16) return false;
    if (a->mma_layout == 3) return true;
    if (a->chunk != 1 || a->head_dim != 64) return false;
    if (a->key_count < 0) return a->B <= kDirRaggedMaxRows;
    const bool mid = a->key_count > kDirMidKeysLo && a->key_count <= kDirMidKeysHi;
    return a->key_count > 0 && a->key_count <= (int64_t)kDirAutoMaxKeys * a->B && !mid;
}

Plan make_direct_plan(const sdl_attn_args* a) {
    Plan pl;
    pl.tc = true;
    pl.direct = true;
    // kv heads per CTA: one unless kv_heads_per_cta asks for more (the
    // most dividing Hkv and kDirWarps up to it).  Reading a token row's
    // heads together measured no faster (C2 decode 33.9 against 34.4 us,
    // long-context decode 65.1 against 62.8 us).
    for (int gc = std::min(a->Hkv, kDirWarps); gc >= 1; --gc) {
        if (a->Hkv % gc || kDirWarps % gc) continue;
        if (gc > std::max(1, a->kv_heads_per_cta)) continue;
        pl.g_cta = gc;
        break;
    }
    pl.kvgroups = a->Hkv / pl.g_cta;
    pl.wpg = kDirWarps / pl.g_cta;
    const int max_pages = std::max(1, (a->max_limit + kPage - 1) / kPage);
    const long base_ctas = (long)a->B * pl.kvgroups;
    const int occ = a->key_count > 0 ? direct_occupancy(a->head_dim, a->dtype) : 0;
    finish_split_plan(a, pl, split_pages(a, base_ctas, max_pages, occ, kRaggedSplitDivDirect), max_pages, 1);
    return pl;
}

Plan make_plan(const sdl_attn_args* a) {
    if (umma_applicable(a)) return make_umma_plan(a);
    if (direct_applicable(a)) return make_direct_plan(a);
    if (rows_applicable(a)) return make_rows_plan(a);
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
    const int ncl = pl.g_cta * pl.wpg * pl.ntg * 8;  // query columns of one CTA
    const int part_bytes = ncl * (a->head_dim + 4) * 4 + 2 * ncl * 4;
    pl.ring_bytes = std::max(kStages * pl.stage_bytes, part_bytes);
    pl.smem = (size_t)pl.ring_bytes + 1024 + (2 * kStages + 2) * sizeof(uint64_t);
    const int max_pages = std::max(1, (a->max_limit + kPage - 1) / kPage);
    const long base_ctas = (long)a->B * pl.ncoltiles * pl.kvgroups;
    const int occ = a->key_count > 0
                        ? tc_occupancy(a->head_dim, pl.ntg, a->dtype, pl.smem, (pl.g_cta * pl.wpg + 1) * 32) : 0;
    const int pps = split_pages(a, base_ctas, max_pages, occ);
    // On-chip merge (opt-in): the row's splits are one cluster of at most
    // kMaxClusterSplits CTAs, which must fit the GPU's cluster occupancy.
    // A cluster is scheduled whole, so the idle splits of short rows hold
    // slots: on ragged batches the workspace merge is faster.
    if (a->cluster_merge) {
        int p2 = pps;
        if (a->pages_per_split <= 0) p2 = std::max(pps, (max_pages + kMaxClusterSplits - 1) / kMaxClusterSplits);
        const int ns = (max_pages + p2 - 1) / p2;
        if (ns > 1 && ns <= kMaxClusterSplits &&
            tc_cluster_fits(a->head_dim, pl.ntg, a->dtype, ns, pl.smem, (pl.g_cta * pl.wpg + 1) * 32)) {
            pl.cluster = true;
            pl.pps = p2;
            pl.nsplit = ns;
            pl.ws_bytes = 0;
            return pl;
        }
    }
    finish_split_plan(a, pl, pps, max_pages, 1);
    return pl;
}

template <int HD, int NTG, typename T>
int launch_tc_inst(const CUtensorMap& mk, const CUtensorMap& mv, const TcParams& tp, const Plan& pl, cudaStream_t st) {
    auto kern = attn_tc_kernel<HD, NTG, T>;
    int rc = tc_configure<HD, NTG, T>(pl.smem);
    if (rc != SDL_OK) return rc;
    dim3 grid(pl.nsplit, pl.ncoltiles * pl.kvgroups, tp.B);
    dim3 block((pl.g_cta * pl.wpg + 1) * 32);
    cudaError_t e = pl.cluster ? sdl::launch_pdl_cluster(kern, grid, block, pl.smem, st, (unsigned)pl.nsplit, mk, mv, tp)
                               : sdl::launch_pdl(kern, grid, block, pl.smem, st, mk, mv, tp);
    if (e != cudaSuccess) return sdl::fail(SDL_ERR_CUDA, cudaGetErrorString(e));
    return sdl::check_launch("attn_tc_kernel");
}

template <int HD, typename T>
int launch_rows_inst(const CUtensorMap& mk, const CUtensorMap& mv, const TcParams& tp, const Plan& pl, cudaStream_t st) {
    auto kern = attn_rows_kernel<HD, T>;
    int rc = rows_configure<HD, T>(pl.smem);
    if (rc != SDL_OK) return rc;
    dim3 grid(pl.nsplit, pl.ncoltiles * pl.kvgroups, tp.B);
    cudaError_t e = sdl::launch_pdl(kern, grid, dim3((pl.wpg + 1) * 32), pl.smem, st, mk, mv, tp);
    if (e != cudaSuccess) return sdl::fail(SDL_ERR_CUDA, cudaGetErrorString(e));
    return sdl::check_launch("attn_rows_kernel");
}

template <typename T>
int launch_rows_dtype(int hd, const CUtensorMap& mk, const CUtensorMap& mv, const TcParams& tp, const Plan& pl,
                      cudaStream_t st) {
    return hd == 64 ? launch_rows_inst<64, T>(mk, mv, tp, pl, st) : launch_rows_inst<128, T>(mk, mv, tp, pl, st);
}

template <typename T>
int launch_direct_dtype(int hd, const TcParams& tp, const Plan& pl, cudaStream_t st) {
    const dim3 grid(pl.nsplit, pl.kvgroups, tp.B), block(kDirWarps * 32);
    const cudaError_t e = hd == 64 ? sdl::launch_pdl(attn_direct_kernel<64, T>, grid, block, 0, st, tp)
                                   : sdl::launch_pdl(attn_direct_kernel<128, T>, grid, block, 0, st, tp);
    if (e != cudaSuccess) return sdl::fail(SDL_ERR_CUDA, cudaGetErrorString(e));
    return sdl::check_launch("attn_direct_kernel");
}

template <int HD, typename T>
int launch_umma_inst(const CUtensorMap& mk, const CUtensorMap& mv, const TcParams& tp, const Plan& pl, cudaStream_t st) {
    auto kern = attn_sk_kernel<HD, T>;
    static bool configured = false;
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pl.smem);
        if (e != cudaSuccess) return sdl::fail(SDL_ERR_CUDA, cudaGetErrorString(e));
        configured = true;
    }
    cudaError_t e = sdl::launch_pdl(kern, dim3(pl.nsplit), dim3(kUThreads), pl.smem, st, mk, mv, tp);
    if (e != cudaSuccess) return sdl::fail(SDL_ERR_CUDA, cudaGetErrorString(e));
    int rc = sdl::check_launch("attn_sk_kernel");
    if (rc != SDL_OK) return rc;
    const int rows = tp.B * tp.Hkv * tp.chunk * tp.ratio;
    e = sdl::launch_pdl(attn_sk_combine_kernel, dim3((rows + 3) / 4), dim3(128), 0, st, tp, HD);
    if (e != cudaSuccess) return sdl::fail(SDL_ERR_CUDA, cudaGetErrorString(e));
    return sdl::check_launch("attn_sk_combine_kernel");
}

template <typename T>
int launch_umma_dtype(int hd, const CUtensorMap& mk, const CUtensorMap& mv, const TcParams& tp, const Plan& pl,
                      cudaStream_t st) {
    if (hd == 64) return launch_umma_inst<64, T>(mk, mv, tp, pl, st);
    return launch_umma_inst<128, T>(mk, mv, tp, pl, st);
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
    if (a->k_new) {
        const int es = sdl::dtype_bytes(a->dtype);
        const int64_t sb = a->new_row_stride * es;
        if (!a->k_pool || !a->v_new || a->new_row_stride < (int64_t)a->Hkv * a->head_dim || sb % 4 ||
            reinterpret_cast<uintptr_t>(a->k_new) % 4 || reinterpret_cast<uintptr_t>(a->v_new) % 4 ||
            reinterpret_cast<uintptr_t>(a->k_pool) % 4 || reinterpret_cast<uintptr_t>(a->v_pool) % 4 ||
            ((int64_t)a->Hkv * a->head_dim * es) % 4)
            return sdl::fail(SDL_ERR_INVALID, "sdl_paged_attention: bad fused-append arguments (k_new/v_new need a "
                                              "paged pool, rows of at least Hkv*head_dim and 4-byte alignment)");
    }
    if ((a->rope_cos != nullptr) != (a->rope_sin != nullptr) ||
        (a->rope_cos && (!a->k_new || a->rope_stride < a->head_dim || a->head_dim % 2)))
        return sdl::fail(SDL_ERR_INVALID, "sdl_paged_attention: bad RoPE arguments (rope_cos and rope_sin together, "
                                          "with k_new and rows of at least head_dim)");
    return SDL_OK;
}

// Whether the mma.sync kernel may write the new K/V rows itself (16-byte pieces).
bool append_fusable(const sdl_attn_args* a) {
    const int64_t sb = a->new_row_stride * sdl::dtype_bytes(a->dtype);
    auto al16 = [](const void* q) { return reinterpret_cast<uintptr_t>(q) % 16 == 0; };
    return a->k_new && al16(a->k_new) && al16(a->v_new) && al16(a->k_pool) && al16(a->v_pool) && sb % 16 == 0;
}

// Whether plan `pl` applies RoPE inside the launch: the mma.sync kernels
// (keys or query rows on M, TMA-fed or register-direct) that store the new
// rows themselves, over 16-byte aligned cos / sin rows (K pieces are rotated
// as 16-byte pieces).
bool rope_fusable(const sdl_attn_args* a, const Plan& pl) {
    auto al16 = [](const void* q) { return reinterpret_cast<uintptr_t>(q) % 16 == 0; };
    const int64_t rb = a->rope_stride * sdl::dtype_bytes(a->dtype);
    return a->rope_cos && pl.tc && !pl.umma && append_fusable(a) && al16(a->rope_cos) &&
           al16(a->rope_sin) && rb % 16 == 0;
}

// Separate positional append (paths that do not write inside the kernel).
int launch_append_pos(const sdl_attn_args* a, cudaStream_t st) {
    TcParams tp = {};
    tp.B = a->B; tp.chunk = a->chunk; tp.valid_rows = a->valid_rows; tp.starts = a->starts; tp.rows = a->rows;
    tp.table = a->block_table; tp.width = a->width; tp.capacity = a->capacity; tp.layer = a->layer;
    tp.k_pool = static_cast<char*>(const_cast<void*>(a->k_pool));
    tp.v_pool = static_cast<char*>(const_cast<void*>(a->v_pool));
    tp.k_new = static_cast<const char*>(a->k_new);
    tp.v_new = static_cast<const char*>(a->v_new);
    const int es = sdl::dtype_bytes(a->dtype);
    tp.new_stride = a->new_row_stride * es;
    tp.err = a->err;
    const int rows = a->B * a->chunk;
    kv_append_pos_kernel<<<(rows + 3) / 4, 128, 0, st>>>(tp, a->Hkv * a->head_dim * es, a->block_size);
    return sdl::check_launch("kv_append_pos_kernel");
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

extern "C" int sdl_attention_kernel(const sdl_attn_args* args) {
    if (validate(args) != SDL_OK) return -1;
    sdl_attn_args tmp = *args;
    tmp.workspace = nullptr;
    tmp.workspace_bytes = 0;
    const Plan pl = make_plan(&tmp);
    return !pl.tc ? 0 : pl.umma ? 2 : pl.rows ? 3 : pl.direct ? 4 : 1;
}

extern "C" int sdl_attention_fuses_rope(const sdl_attn_args* args) {
    if (validate(args) != SDL_OK) return -1;
    sdl_attn_args tmp = *args;
    tmp.workspace = nullptr;
    tmp.workspace_bytes = 0;
    return rope_fusable(&tmp, make_plan(&tmp)) ? 1 : 0;
}

extern "C" int sdl_attention_launches(const sdl_attn_args* args) {
    if (validate(args) != SDL_OK) return -1;
    if (args->B == 0) return 0;
    sdl_attn_args tmp = *args;
    tmp.workspace = nullptr;
    tmp.workspace_bytes = 0;
    const Plan pl = make_plan(&tmp);
    const bool fused_append = tmp.k_new && pl.tc && !pl.umma && append_fusable(&tmp);
    int n = (tmp.k_new && !fused_append) ? 1 : 0;
    if (!pl.tc) return n + 1;
    return n + 1 + ((pl.umma || (pl.nsplit > 1 && !pl.cluster)) ? 1 : 0);
}

extern "C" int sdl_paged_attention(const sdl_attn_args* a, void* stream) {
    int rc = validate(a);
    if (rc != SDL_OK) return rc;
    if (a->B == 0) return SDL_OK;
    cudaStream_t st = sdl::as_stream(stream);
    const int ratio = a->Hq / a->Hkv;
    Plan pl = make_plan(a);
    // The mma.sync kernel stores the new rows itself (16-byte pieces).  The
    // tcgen05 kernel does not: a store + proxy fence inside its producer
    // stalls a deep TMA pipeline longer than a separate append launch costs.
    const bool fused_append = a->k_new && pl.tc && !pl.umma && append_fusable(a);
    if (a->rope_cos && !rope_fusable(a, pl))
        return sdl::fail(SDL_ERR_UNSUPPORTED, "sdl_paged_attention: this plan cannot apply RoPE inside the launch");
    if (a->k_new && !fused_append && (rc = launch_append_pos(a, st)) != SDL_OK) return rc;
    if (pl.tc) {
        if (pl.ws_bytes > 0 && (!a->workspace || a->workspace_bytes < pl.ws_bytes))
            return sdl::fail(SDL_ERR_WORKSPACE, "sdl_paged_attention: workspace too small");
        CUtensorMap mk = {}, mv = {};
        if (pl.direct) {
            // plain loads: no tensor maps
        } else if (a->k_pool) {
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
        tp.ring_bytes = pl.ring_bytes;
        tp.stages = pl.stages;
        tp.cluster = pl.cluster ? 1 : 0;
        tp.scale_log2 = a->scale * 1.4426950408889634f;
        tp.o_part = a->workspace;
        tp.ml_part = a->workspace ? a->workspace + (size_t)a->B * pl.nsplit * a->chunk * a->Hq * a->head_dim : nullptr;
        tp.sk_table = nullptr;
        tp.k_pool = tp.v_pool = nullptr;
        tp.k_new = tp.v_new = nullptr;
        tp.new_stride = 0;
        tp.k_src = static_cast<const char*>(a->k_pool ? a->k_pool : a->k_dense);
        tp.v_src = static_cast<const char*>(a->k_pool ? a->v_pool : a->v_dense);
        tp.overlap = a->overlap_layers ? 1 : 0;
        tp.rope_cos = static_cast<const char*>(a->rope_cos);
        tp.rope_sin = static_cast<const char*>(a->rope_sin);
        tp.rope_stride = a->rope_stride;
        if (fused_append) {
            tp.k_pool = static_cast<char*>(const_cast<void*>(a->k_pool));
            tp.v_pool = static_cast<char*>(const_cast<void*>(a->v_pool));
            tp.k_new = static_cast<const char*>(a->k_new);
            tp.v_new = static_cast<const char*>(a->v_new);
            tp.new_stride = a->new_row_stride * sdl::dtype_bytes(a->dtype);
        }
        if (pl.umma) {
            const int npairs = a->B * a->Hkv;
            const size_t slots = (size_t)(pl.nsplit + npairs) * a->chunk * ratio;
            tp.sk_table = reinterpret_cast<int4*>(a->workspace);
            tp.o_part = a->workspace + sk_header_bytes(npairs) / sizeof(float);
            tp.ml_part = tp.o_part + slots * a->head_dim;
        }
        tp.err = a->err;
        if (pl.umma) {
            if (a->dtype == SDL_BF16) rc = launch_umma_dtype<__nv_bfloat16>(a->head_dim, mk, mv, tp, pl, st);
            else rc = launch_umma_dtype<__half>(a->head_dim, mk, mv, tp, pl, st);
        } else if (pl.direct) {
            if (a->dtype == SDL_BF16) rc = launch_direct_dtype<__nv_bfloat16>(a->head_dim, tp, pl, st);
            else rc = launch_direct_dtype<__half>(a->head_dim, tp, pl, st);
        } else if (pl.rows) {
            if (a->dtype == SDL_BF16) rc = launch_rows_dtype<__nv_bfloat16>(a->head_dim, mk, mv, tp, pl, st);
            else rc = launch_rows_dtype<__half>(a->head_dim, mk, mv, tp, pl, st);
        } else if (a->dtype == SDL_BF16) {
            rc = launch_tc_dtype<__nv_bfloat16>(a->head_dim, pl.ntg, mk, mv, tp, pl, st);
        } else {
            rc = launch_tc_dtype<__half>(a->head_dim, pl.ntg, mk, mv, tp, pl, st);
        }
        if (rc != SDL_OK) return rc;
        if (pl.nsplit > 1 && !pl.umma && !pl.cluster) {
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
    // The plan is made against the static array, so an automatic split
    // size grows until the partials fit it; only a plan that cannot shrink
    // (an explicit pages_per_split, the tcgen05 kernel) can still need more.
    float* scratch = nullptr;
    if ((rc = noalloc_scratch(&scratch)) != SDL_OK) return rc;
    sdl_attn_args a = *args;
    a.workspace = scratch;
    a.workspace_bytes = kNoAllocScratchBytes;
    const size_t need = make_plan(&a).ws_bytes;
    if (need > kNoAllocScratchBytes) {
        char msg[256];
        snprintf(msg, sizeof(msg),
                 "sdl_paged_attention_noalloc: this call needs %zu bytes of split-K scratch, more than the "
                 "%zu-byte static scratch; pass a workspace to sdl_paged_attention instead",
                 need, kNoAllocScratchBytes);
        return sdl::fail(SDL_ERR_WORKSPACE, msg);
    }
    return sdl_paged_attention(&a, stream);
}

extern "C" int sdl_paged_decode(const sdl_attn_args* args, void* stream) {
    if (args && args->chunk != 1) return sdl::fail(SDL_ERR_INVALID, "sdl_paged_decode: chunk must be 1");
    return sdl_paged_attention(args, stream);
}

extern "C" int sdl_paged_verify(const sdl_attn_args* args, void* stream) { return sdl_paged_attention(args, stream); }

extern "C" int sdl_prefill_chunk(const sdl_attn_args* args, void* stream) { return sdl_paged_attention(args, stream); }
