// Paged-KV storage kernels: LIFO free list, batched reserve (allocation +
// slot mapping), vectorised K/V append, ordered rewind/clear and the
// device-side commit of a speculative round.
//
// Ordering contract.  The reference allocator is a Python list used as a
// stack (engine/kv.py:52,68: pop() from the end, free() appends); blocks are
// allocated lazily by per-token writes in sequence-major, token-minor order
// (engine/model.py:143-145,184-187, engine/qwen.py:124-125,161-164,191-194);
// truncate frees a table's tail from the end (engine/kv.py:160-161) and clear
// frees it from the front (engine/kv.py:167-168).  Every kernel below keeps
// exactly that push/pop order, so block tables match the reference
// bit-for-bit.  Metadata kernels run as one CTA: they touch a few hundred
// ints per round and are launch-latency bound, not bandwidth bound.
#include "sdl_common.cuh"

#include <cstdio>

namespace sdl {
static thread_local std::string g_last_error;
void set_last_error(const std::string& msg) { g_last_error = msg; }
}  // namespace sdl

extern "C" const char* sdl_version(void) { return "sdl_b200 0.1.0 (sm_100a)"; }
extern "C" const char* sdl_last_error(void) { return sdl::g_last_error.c_str(); }

// ------------------------------------------------------------ free list ops
SDL_DEV void push_block(const sdl_kv_meta& m, int32_t blk, int32_t& top) {
    if (blk < 0 || blk >= m.capacity) { sdl_raise(m.err, SDL_DEVERR_BAD_INDEX); return; }
    if (m.is_free[blk]) return;  // idempotent double free
    m.free_stack[top++] = blk;
    m.is_free[blk] = 1;
}

SDL_DEV bool row_ok(const sdl_kv_meta& m, int32_t row) { return row >= 0 && row < m.max_rows; }

// Rewind one row to new_len: free blocks past ceil(new_len/bs), last first.
SDL_DEV void seq_truncate(const sdl_kv_meta& m, int32_t row, int32_t new_len, int32_t& top) {
    const int32_t bs = m.block_size;
    int32_t keep_b = new_len <= 0 ? 0 : (new_len + bs - 1) / bs;
    int32_t nb = m.num_blocks[row];
    int32_t* tab = m.block_table + (int64_t)row * m.width;
    while (nb > keep_b) {
        --nb;
        push_block(m, tab[nb], top);
        tab[nb] = -1;
    }
    m.num_blocks[row] = nb;
    m.seq_lens[row] = new_len < 0 ? 0 : new_len;
}

// Drop one row: free every block front to back.
SDL_DEV void seq_clear(const sdl_kv_meta& m, int32_t row, int32_t& top) {
    int32_t nb = m.num_blocks[row];
    int32_t* tab = m.block_table + (int64_t)row * m.width;
    for (int32_t i = 0; i < nb; ++i) {
        push_block(m, tab[i], top);
        tab[i] = -1;
    }
    m.num_blocks[row] = 0;
    m.seq_lens[row] = 0;
}

// Back position `pos` of `row` with a block (popping when needed), extend the
// length, return its slot or -1 on exhaustion / overflow.
SDL_DEV int32_t seq_extend_one(const sdl_kv_meta& m, int32_t row, int32_t pos, int32_t& top) {
    const int32_t bs = m.block_size;
    int32_t need_b = pos / bs + 1;
    if (need_b > m.width) { sdl_raise(m.err, SDL_DEVERR_TABLE_OVERFLOW); return -1; }
    int32_t nb = m.num_blocks[row];
    int32_t* tab = m.block_table + (int64_t)row * m.width;
    while (nb < need_b) {
        if (top <= 0) { sdl_raise(m.err, SDL_DEVERR_EXHAUSTED); m.num_blocks[row] = nb; return -1; }
        int32_t blk = m.free_stack[--top];
        m.is_free[blk] = 0;
        tab[nb++] = blk;
    }
    m.num_blocks[row] = nb;
    if (m.seq_lens[row] <= pos) m.seq_lens[row] = pos + 1;
    return tab[pos / bs] * bs + pos % bs;
}

// ------------------------------------------------------------------ kernels
__global__ void block_init_kernel(int32_t* stack, int32_t* top, uint8_t* is_free, int32_t cap) {
    for (int32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < cap; i += gridDim.x * blockDim.x) {
        stack[i] = i;
        is_free[i] = 1;
    }
    if (blockIdx.x == 0 && threadIdx.x == 0) *top = cap;
}

__global__ void block_alloc_kernel(int32_t* stack, int32_t* top_p, uint8_t* is_free, int32_t n,
                                   int32_t* out, int32_t* err) {
    if (threadIdx.x != 0) return;
    int32_t top = *top_p;
    if (top < n) {
        sdl_raise(err, SDL_DEVERR_EXHAUSTED);
        for (int32_t k = 0; k < n; ++k) out[k] = -1;
        return;
    }
    for (int32_t k = 0; k < n; ++k) {
        int32_t blk = stack[--top];
        is_free[blk] = 0;
        out[k] = blk;
    }
    *top_p = top;
}

__global__ void block_free_kernel(int32_t* stack, int32_t* top_p, uint8_t* is_free, int32_t cap,
                                  int32_t n, const int32_t* blocks, int32_t* err) {
    if (threadIdx.x != 0) return;
    int32_t top = *top_p;
    for (int32_t k = 0; k < n; ++k) {
        int32_t blk = blocks[k];
        if (blk < 0 || blk >= cap) { sdl_raise(err, SDL_DEVERR_BAD_INDEX); continue; }
        if (is_free[blk]) continue;
        stack[top++] = blk;
        is_free[blk] = 1;
    }
    *top_p = top;
}

// New blocks a reserve of [start, start+count) needs for `row`; flags errors.
SDL_DEV int32_t reserve_need(const sdl_kv_meta& m, int32_t row, int32_t st, int32_t cnt, int32_t* bad) {
    if (cnt <= 0) return 0;
    if (!row_ok(m, row) || st < 0) { atomicOr(bad, SDL_DEVERR_BAD_INDEX); return 0; }
    int64_t end = (int64_t)st + cnt;
    int64_t nb_need = (end + m.block_size - 1) / m.block_size;
    if (nb_need > m.width) { atomicOr(bad, SDL_DEVERR_TABLE_OVERFLOW); return 0; }
    int32_t nb = m.num_blocks[row];
    return nb_need > nb ? (int32_t)(nb_need - nb) : 0;
}

__global__ void __launch_bounds__(1024) kv_reserve_kernel(sdl_kv_meta m, int32_t n, const int32_t* rows,
                                                          const int32_t* starts, const int32_t* counts,
                                                          int32_t* slots) {
    __shared__ int32_t ws[32];
    __shared__ int32_t s_bad;
    __shared__ int32_t s_top;
    if (threadIdx.x == 0) { s_bad = 0; s_top = *m.free_top; }
    __syncthreads();
    const int32_t bs = m.block_size;

    // Pass 0: validate and total the new blocks.
    int32_t tot_new = 0;
    for (int32_t base = 0; base < n; base += blockDim.x) {
        int32_t i = base + threadIdx.x;
        int32_t need = 0;
        if (i < n) need = reserve_need(m, rows[i], starts[i], counts[i], &s_bad);
        tot_new += block_sum<int32_t>(need, ws);
    }
    __syncthreads();
    int32_t bad = s_bad;
    if (!bad && tot_new > s_top) bad = SDL_DEVERR_EXHAUSTED;

    int32_t new_carry = 0, tok_carry = 0;
    for (int32_t base = 0; base < n; base += blockDim.x) {
        int32_t i = base + threadIdx.x;
        int32_t row = 0, st = 0, cnt = 0, need = 0;
        if (i < n) {
            row = rows[i]; st = starts[i]; cnt = counts[i] > 0 ? counts[i] : 0;
            if (!bad) need = reserve_need(m, row, st, cnt, &s_bad);
        }
        int32_t tnew, ttok;
        int32_t off_new = block_exclusive_scan<int32_t>(need, ws, &tnew) + new_carry;
        int32_t off_tok = block_exclusive_scan<int32_t>(cnt, ws, &ttok) + tok_carry;
        if (i < n && cnt > 0) {
            if (bad) {
                for (int32_t j = 0; j < cnt; ++j) slots[off_tok + j] = -1;
            } else {
                int32_t* tab = m.block_table + (int64_t)row * m.width;
                int32_t nb = m.num_blocks[row];
                for (int32_t k = 0; k < need; ++k) {
                    int32_t blk = m.free_stack[s_top - 1 - (off_new + k)];
                    tab[nb + k] = blk;
                    m.is_free[blk] = 0;
                }
                m.num_blocks[row] = nb + need;
                int32_t end = st + cnt;
                if (m.seq_lens[row] < end) m.seq_lens[row] = end;
                for (int32_t j = 0; j < cnt; ++j) {
                    int32_t pos = st + j;
                    slots[off_tok + j] = tab[pos / bs] * bs + pos % bs;
                }
            }
        }
        new_carry += tnew;
        tok_carry += ttok;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        if (bad) atomicOr(m.err, bad);
        else *m.free_top = s_top - tot_new;
    }
}

// One thread per 16-byte (or element-sized) chunk of a K or V token row.
template <typename W>
__global__ void kv_append_kernel(char* __restrict__ kpool, char* __restrict__ vpool, int64_t layer_off,
                                 int64_t pool_slots, int32_t row_bytes, int32_t ntok,
                                 const int32_t* __restrict__ slots, const char* __restrict__ ksrc,
                                 const char* __restrict__ vsrc, int64_t src_stride, int32_t* err) {
    pdl_launch_dependents();  // the attention launch may start its prologue now
    const int32_t chunks = row_bytes / (int32_t)sizeof(W);
    const int64_t total = (int64_t)ntok * chunks * 2;
    for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
         idx += (int64_t)gridDim.x * blockDim.x) {
        int32_t c = (int32_t)(idx % chunks);
        int64_t rest = idx / chunks;
        int32_t which = (int32_t)(rest & 1);
        int32_t t = (int32_t)(rest >> 1);
        int32_t slot = slots[t];
        if (slot < 0) continue;
        if ((int64_t)slot >= pool_slots) { sdl_raise(err, SDL_DEVERR_BAD_SLOT); continue; }
        const W* src = reinterpret_cast<const W*>((which ? vsrc : ksrc) + (int64_t)t * src_stride);
        W* dst = reinterpret_cast<W*>((which ? vpool : kpool) + layer_off + (int64_t)slot * row_bytes);
        dst[c] = src[c];
    }
}

// Per-sequence truncate / clear in list order.  Pass 0 counts each row's
// pushes, a block scan turns them into stack offsets, pass 1 writes them.
__global__ void __launch_bounds__(1024) kv_release_kernel(sdl_kv_meta m, int32_t n, const int32_t* rows,
                                                          const int32_t* new_lens, const int32_t* flags) {
    __shared__ int32_t ws[32];
    __shared__ int32_t s_top;
    if (threadIdx.x == 0) s_top = *m.free_top;
    __syncthreads();
    const int32_t bs = m.block_size;
    int32_t carry = 0;
    for (int32_t base = 0; base < n; base += blockDim.x) {
        int32_t i = base + threadIdx.x;
        int32_t row = -1, nb = 0, keep_b = 0, cnt = 0, f = 0, nl = 0;
        bool do_trunc = false;
        if (i < n) {
            row = rows[i];
            f = flags ? flags[i] : SDL_REL_TRUNCATE;
            nl = new_lens ? new_lens[i] : 0;
            if (!row_ok(m, row)) {
                sdl_raise(m.err, SDL_DEVERR_BAD_INDEX);
                row = -1;
            } else {
                nb = m.num_blocks[row];
                keep_b = nb;
                int32_t len = m.seq_lens[row];
                do_trunc = (f & SDL_REL_TRUNCATE) && (!(f & SDL_REL_ONLY_IF_LONGER) || len > nl);
                if (do_trunc) {
                    int32_t kb = nl <= 0 ? 0 : (nl + bs - 1) / bs;
                    if (kb < nb) keep_b = kb;
                }
                const int32_t* tab = m.block_table + (int64_t)row * m.width;
                for (int32_t k = keep_b; k < nb; ++k) {
                    int32_t blk = tab[k];
                    cnt += (blk >= 0 && blk < m.capacity && !m.is_free[blk]) ? 1 : 0;
                }
                if (f & SDL_REL_CLEAR)
                    for (int32_t k = 0; k < keep_b; ++k) {
                        int32_t blk = tab[k];
                        cnt += (blk >= 0 && blk < m.capacity && !m.is_free[blk]) ? 1 : 0;
                    }
            }
        }
        int32_t tot;
        int32_t off = block_exclusive_scan<int32_t>(cnt, ws, &tot) + carry;
        if (row >= 0) {
            int32_t top = s_top + off;
            int32_t* tab = m.block_table + (int64_t)row * m.width;
            for (int32_t k = nb - 1; k >= keep_b; --k) {
                push_block(m, tab[k], top);
                tab[k] = -1;
            }
            if (do_trunc) {
                m.num_blocks[row] = keep_b;
                m.seq_lens[row] = nl < 0 ? 0 : nl;
            }
            if (f & SDL_REL_CLEAR) {
                for (int32_t k = 0; k < keep_b; ++k) {
                    push_block(m, tab[k], top);
                    tab[k] = -1;
                }
                m.num_blocks[row] = 0;
                m.seq_lens[row] = 0;
            }
        }
        carry += tot;
    }
    __syncthreads();
    if (threadIdx.x == 0) *m.free_top = s_top + carry;
}

// Commit of one speculative round.  Lane 0 of warp 0 walks the target cache,
// lane 0 of warp 1 the draft cache; each walks the sequences in list order.
__global__ void spec_commit_kernel(sdl_kv_meta tgt, sdl_kv_meta drf, int32_t has_draft, int32_t n,
                                   const int32_t* rows, const int32_t* n_out, const int32_t* tokens,
                                   int32_t tok_stride, const int32_t* remaining, int32_t eos,
                                   const int32_t* starts, int32_t* k_out, int32_t* flags_out,
                                   int32_t* catchup_slot, const int32_t* n_valid) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane != 0 || warp > 1) return;
    const bool is_target = (warp == 0);
    if (!is_target && !has_draft) return;
    const sdl_kv_meta& m = is_target ? tgt : drf;
    // rows past *n_valid pad a captured batch: they are not committed
    if (n_valid != nullptr) n = min(n, max(0, *n_valid));
    int32_t top = *m.free_top;
    for (int32_t b = 0; b < n; ++b) {
        int32_t row = rows[b];
        int32_t rem = remaining[b];
        int32_t k = n_out[b] < rem ? n_out[b] : rem;
        if (k < 0) k = 0;
        int32_t eos_hit = 0;
        if (eos >= 0) {
            for (int32_t i = 0; i < k; ++i) {
                if (tokens[(int64_t)b * tok_stride + i] == eos) { k = i; eos_hit = 1; break; }
            }
        }
        int32_t fin = (eos_hit || k == 0 || k >= rem) ? 1 : 0;
        int32_t keep = starts[b] + k;
        if (!row_ok(m, row)) {
            sdl_raise(m.err, SDL_DEVERR_BAD_INDEX);
            if (is_target) { k_out[b] = k; flags_out[b] = fin | (eos_hit << 1); }
            else catchup_slot[b] = -1;
            continue;
        }
        if (is_target) {
            if (k > 0) seq_truncate(m, row, keep, top);
            if (fin) seq_clear(m, row, top);
            k_out[b] = k;
            flags_out[b] = fin | (eos_hit << 1);
        } else {
            int32_t slot = -1;
            if (k > 0) {
                int32_t d_len = m.seq_lens[row];
                if (d_len > keep) {
                    seq_truncate(m, row, keep, top);
                } else if (d_len < keep) {
                    if (keep - d_len != 1) sdl_raise(m.err, SDL_DEVERR_BAD_INDEX);
                    slot = seq_extend_one(m, row, d_len, top);
                }
            }
            if (fin) { seq_clear(m, row, top); slot = -1; }
            catchup_slot[b] = slot;
        }
    }
    *m.free_top = top;
}

// --------------------------------------------------------------- C entries
extern "C" int sdl_block_init(int32_t* free_stack, int32_t* free_top, uint8_t* is_free, int32_t capacity,
                              void* stream) {
    if (!free_stack || !free_top || !is_free || capacity < 1) return sdl::fail(SDL_ERR_INVALID, "sdl_block_init: bad args");
    int blocks = (capacity + 255) / 256;
    if (blocks > 4096) blocks = 4096;
    block_init_kernel<<<blocks, 256, 0, sdl::as_stream(stream)>>>(free_stack, free_top, is_free, capacity);
    return sdl::check_launch("block_init_kernel");
}

extern "C" int sdl_block_alloc(int32_t* free_stack, int32_t* free_top, uint8_t* is_free, int32_t capacity,
                               int32_t n, int32_t* out_blocks, int32_t* err, void* stream) {
    if (!free_stack || !free_top || !is_free || n < 0 || (n > 0 && !out_blocks) || n > capacity)
        return sdl::fail(SDL_ERR_INVALID, "sdl_block_alloc: bad args");
    if (n == 0) return SDL_OK;
    block_alloc_kernel<<<1, 32, 0, sdl::as_stream(stream)>>>(free_stack, free_top, is_free, n, out_blocks, err);
    return sdl::check_launch("block_alloc_kernel");
}

extern "C" int sdl_block_free(int32_t* free_stack, int32_t* free_top, uint8_t* is_free, int32_t capacity,
                              int32_t n, const int32_t* blocks, int32_t* err, void* stream) {
    if (!free_stack || !free_top || !is_free || n < 0 || (n > 0 && !blocks))
        return sdl::fail(SDL_ERR_INVALID, "sdl_block_free: bad args");
    if (n == 0) return SDL_OK;
    block_free_kernel<<<1, 32, 0, sdl::as_stream(stream)>>>(free_stack, free_top, is_free, capacity, n, blocks, err);
    return sdl::check_launch("block_free_kernel");
}

static bool meta_ok(const sdl_kv_meta* m) {
    return m && m->block_table && m->num_blocks && m->seq_lens && m->free_stack && m->free_top && m->is_free &&
           m->err && m->capacity > 0 && m->width > 0 && m->max_rows > 0 && m->block_size > 0;
}

extern "C" int sdl_kv_reserve(const sdl_kv_meta* meta, int32_t n, const int32_t* rows, const int32_t* starts,
                              const int32_t* counts, int32_t* slots, void* stream) {
    if (!meta_ok(meta) || n < 0 || (n > 0 && (!rows || !starts || !counts || !slots)))
        return sdl::fail(SDL_ERR_INVALID, "sdl_kv_reserve: bad args");
    if (n == 0) return SDL_OK;
    kv_reserve_kernel<<<1, 1024, 0, sdl::as_stream(stream)>>>(*meta, n, rows, starts, counts, slots);
    return sdl::check_launch("kv_reserve_kernel");
}

extern "C" int sdl_kv_append(void* k_pool, void* v_pool, int32_t dtype, int32_t num_layers, int32_t capacity,
                             int32_t block_size, int32_t row_elems, int32_t layer, int32_t num_tokens,
                             const int32_t* slots, const void* k_src, const void* v_src, int64_t src_row_stride,
                             int32_t* err, void* stream) {
    if (!k_pool || !v_pool || num_layers < 1 || capacity < 1 || block_size < 1 || row_elems < 1 || layer < 0 ||
        layer >= num_layers || num_tokens < 0 || (num_tokens > 0 && (!slots || !k_src || !v_src)) ||
        src_row_stride < row_elems || (dtype != SDL_F32 && dtype != SDL_BF16 && dtype != SDL_F16))
        return sdl::fail(SDL_ERR_INVALID, "sdl_kv_append: bad args");
    if (num_tokens == 0) return SDL_OK;
    const int es = sdl::dtype_bytes(dtype);
    const int32_t row_bytes = row_elems * es;
    const int64_t src_stride = src_row_stride * es;
    const int64_t pool_slots = (int64_t)capacity * block_size;
    const int64_t layer_off = (int64_t)layer * pool_slots * row_bytes;
    auto aligned = [](const void* p, int a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; };
    cudaStream_t st = sdl::as_stream(stream);
    char* kp = static_cast<char*>(k_pool);
    char* vp = static_cast<char*>(v_pool);
    const char* ks = static_cast<const char*>(k_src);
    const char* vs = static_cast<const char*>(v_src);
    int threads = 256;
    if (row_bytes % 16 == 0 && src_stride % 16 == 0 && aligned(kp, 16) && aligned(vp, 16) && aligned(ks, 16) &&
        aligned(vs, 16)) {
        int64_t total = (int64_t)num_tokens * (row_bytes / 16) * 2;
        int blocks = (int)((total + threads - 1) / threads);
        if (blocks > 8192) blocks = 8192;
        kv_append_kernel<uint4><<<blocks, threads, 0, st>>>(kp, vp, layer_off, pool_slots, row_bytes, num_tokens,
                                                            slots, ks, vs, src_stride, err);
    } else if (row_bytes % 4 == 0 && src_stride % 4 == 0 && aligned(ks, 4) && aligned(vs, 4)) {
        int64_t total = (int64_t)num_tokens * (row_bytes / 4) * 2;
        int blocks = (int)((total + threads - 1) / threads);
        if (blocks > 8192) blocks = 8192;
        kv_append_kernel<uint32_t><<<blocks, threads, 0, st>>>(kp, vp, layer_off, pool_slots, row_bytes, num_tokens,
                                                               slots, ks, vs, src_stride, err);
    } else {
        int64_t total = (int64_t)num_tokens * (row_bytes / 2) * 2;
        int blocks = (int)((total + threads - 1) / threads);
        if (blocks > 8192) blocks = 8192;
        kv_append_kernel<uint16_t><<<blocks, threads, 0, st>>>(kp, vp, layer_off, pool_slots, row_bytes, num_tokens,
                                                               slots, ks, vs, src_stride, err);
    }
    return sdl::check_launch("kv_append_kernel");
}

extern "C" int sdl_kv_release(const sdl_kv_meta* meta, int32_t n, const int32_t* rows, const int32_t* new_lens,
                              const int32_t* flags, void* stream) {
    if (!meta_ok(meta) || n < 0 || (n > 0 && !rows)) return sdl::fail(SDL_ERR_INVALID, "sdl_kv_release: bad args");
    if (n == 0) return SDL_OK;
    kv_release_kernel<<<1, 1024, 0, sdl::as_stream(stream)>>>(*meta, n, rows, new_lens, flags);
    return sdl::check_launch("kv_release_kernel");
}

extern "C" int sdl_kv_truncate(const sdl_kv_meta* meta, int32_t n, const int32_t* rows, const int32_t* new_lens,
                               void* stream) {
    if (!new_lens) return sdl::fail(SDL_ERR_INVALID, "sdl_kv_truncate: new_lens is NULL");
    return sdl_kv_release(meta, n, rows, new_lens, nullptr, stream);
}

namespace {
int spec_commit_impl(const sdl_kv_meta* target, const sdl_kv_meta* draft, int32_t n, const int32_t* rows,
                     const int32_t* n_out, const int32_t* tokens, int32_t tok_stride, const int32_t* remaining,
                     int32_t eos, const int32_t* starts, int32_t* k_out, int32_t* flags_out, int32_t* catchup_slot,
                     const int32_t* n_valid, void* stream) {
    if (!meta_ok(target) || (draft && !meta_ok(draft)) || n < 0 ||
        (n > 0 && (!rows || !n_out || !tokens || !remaining || !starts || !k_out || !flags_out ||
                   (draft && !catchup_slot))))
        return sdl::fail(SDL_ERR_INVALID, "sdl_spec_commit: bad args");
    if (n == 0) return SDL_OK;
    sdl_kv_meta d = draft ? *draft : *target;
    spec_commit_kernel<<<1, 64, 0, sdl::as_stream(stream)>>>(*target, d, draft ? 1 : 0, n, rows, n_out, tokens,
                                                            tok_stride, remaining, eos, starts, k_out, flags_out,
                                                            catchup_slot, n_valid);
    return sdl::check_launch("spec_commit_kernel");
}
}  // namespace

extern "C" int sdl_spec_commit(const sdl_kv_meta* target, const sdl_kv_meta* draft, int32_t n, const int32_t* rows,
                               const int32_t* n_out, const int32_t* tokens, int32_t tok_stride,
                               const int32_t* remaining, int32_t eos, const int32_t* starts, int32_t* k_out,
                               int32_t* flags_out, int32_t* catchup_slot, void* stream) {
    return spec_commit_impl(target, draft, n, rows, n_out, tokens, tok_stride, remaining, eos, starts, k_out,
                            flags_out, catchup_slot, nullptr, stream);
}

extern "C" int sdl_spec_commit_n(const sdl_kv_meta* target, const sdl_kv_meta* draft, int32_t n,
                                 const int32_t* rows, const int32_t* n_out, const int32_t* tokens,
                                 int32_t tok_stride, const int32_t* remaining, int32_t eos, const int32_t* starts,
                                 int32_t* k_out, int32_t* flags_out, int32_t* catchup_slot,
                                 const int32_t* n_valid, void* stream) {
    if (!n_valid) return sdl::fail(SDL_ERR_INVALID, "sdl_spec_commit_n: n_valid is NULL");
    return spec_commit_impl(target, draft, n, rows, n_out, tokens, tok_stride, remaining, eos, starts, k_out,
                            flags_out, catchup_slot, n_valid, stream);
}

extern "C" int sdl_get_error(int32_t* err_word, int32_t* out_host, int32_t clear, void* stream) {
    if (!err_word || !out_host) return sdl::fail(SDL_ERR_INVALID, "sdl_get_error: bad args");
    cudaStream_t st = sdl::as_stream(stream);
    cudaError_t e = cudaMemcpyAsync(out_host, err_word, sizeof(int32_t), cudaMemcpyDeviceToHost, st);
    if (e != cudaSuccess) return sdl::fail(SDL_ERR_CUDA, cudaGetErrorString(e));
    if (clear) {
        e = cudaMemsetAsync(err_word, 0, sizeof(int32_t), st);
        if (e != cudaSuccess) return sdl::fail(SDL_ERR_CUDA, cudaGetErrorString(e));
    }
    return SDL_OK;
}
