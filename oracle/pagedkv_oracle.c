/*
 * pagedkv_oracle.c -- CPU restatement of the reference's paged-KV hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
 * kernels in libpagedkv.so and the timed CPU baseline of bench.py.  Only the
 * tests, __graft_entry__.smoke() and bench.py's CPU-baseline leg load it; no
 * product code path calls it.
 *
 * What it restates (reference = kjoshiDTX/llm-inference-scheduler, Python):
 *
 *   orc_reshape_and_cache   the scatter loop of PagedKVCache.append_and_fetch
 *                           (mini_engine/paged/block_manager.py:121-131),
 *                           expressed per token through its slot
 *                           (slot = table[pos // bs] * bs + pos % bs).
 *   orc_copy_blocks         BlockManager.copy_block's per-layer copy of one
 *                           block (block_manager.py:65-71), batched over
 *                           (src, dst) pairs.
 *   orc_paged_attention     the gather (block_manager.py:136-141) followed by
 *                           Qwen2Model._attention (mini_engine/model/qwen2.py:
 *                           98-128), with the reference's rounding points for
 *                           16-bit KV: the Q.K^T product is rounded to the KV
 *                           dtype, the scale multiply is rounded again, the
 *                           softmax runs in fp32, the probabilities are cast
 *                           back to the KV dtype before the PV product, and
 *                           the PV product is rounded to the KV dtype.  The
 *                           causal rule is qwen2.py:118-124: new token i of a
 *                           sequence may attend to key j iff j <= num_prior+i.
 *
 * Accumulation: fp32 for 16-bit inputs (PyTorch's CPU opmath type for Half
 * and BFloat16 matmuls), fp64 for fp32 inputs.  The reference's products come
 * from PyTorch 2.11 CPU kernels whose summation order is not specified, so
 * this restatement agrees with the reference's golden vectors to a tolerance
 * (one 16-bit ulp of a score in rare cases), not bit for bit; the append and
 * copy paths are bit-exact.
 *
 * Layouts: pools [num_blocks][block_size][n_kv_heads][head_dim]; q and out
 * [n_tokens][n_q_heads][head_dim]; block_tables [n_seqs][bt_stride] int32.
 * dtype: 0 = fp32, 1 = fp16, 2 = bf16.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

enum { ORC_F32 = 0, ORC_F16 = 1, ORC_BF16 = 2 };

static inline float h2f(uint16_t h) {
    _Float16 x;
    memcpy(&x, &h, 2);
    return (float)x;
}
static inline uint16_t f2h(float f) {
    _Float16 x = (_Float16)f; /* round to nearest even */
    uint16_t h;
    memcpy(&h, &x, 2);
    return h;
}
static inline float b2f(uint16_t b) {
    uint32_t u = (uint32_t)b << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}
static inline uint16_t f2b(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40); /* quiet NaN */
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

static inline float load_el(const void* p, int64_t i, int dt) {
    if (dt == ORC_F32) return ((const float*)p)[i];
    if (dt == ORC_F16) return h2f(((const uint16_t*)p)[i]);
    return b2f(((const uint16_t*)p)[i]);
}
/* round a float to the storage dtype and back (identity for fp32) */
static inline float round_dt(float x, int dt) {
    if (dt == ORC_F16) return h2f(f2h(x));
    if (dt == ORC_BF16) return b2f(f2b(x));
    return x;
}
static inline void store_el(void* p, int64_t i, float x, int dt) {
    if (dt == ORC_F32) ((float*)p)[i] = x;
    else if (dt == ORC_F16) ((uint16_t*)p)[i] = f2h(x);
    else ((uint16_t*)p)[i] = f2b(x);
}
static inline int esize(int dt) { return dt == ORC_F32 ? 4 : 2; }

int orc_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* Returns 0, or -1 if a slot lies outside the pool (nothing is written for it). */
int orc_reshape_and_cache(const void* k, const void* v, int64_t k_row_stride, int64_t v_row_stride,
                          void* k_pool, void* v_pool, const int64_t* slot_mapping, int n_tokens,
                          int num_blocks, int block_size, int n_kv_heads, int head_dim, int dtype) {
    const int64_t row = (int64_t)n_kv_heads * head_dim * esize(dtype);
    const int64_t n_slots = (int64_t)num_blocks * block_size;
    int bad = 0;
    for (int t = 0; t < n_tokens; ++t) {
        const int64_t s = slot_mapping[t];
        if (s < 0) continue; /* padding token */
        if (s >= n_slots) { bad = 1; continue; }
        memcpy((char*)k_pool + s * row, (const char*)k + (int64_t)t * k_row_stride * esize(dtype), row);
        memcpy((char*)v_pool + s * row, (const char*)v + (int64_t)t * v_row_stride * esize(dtype), row);
    }
    return bad ? -1 : 0;
}

/* pairs: [n_pairs][2] (src, dst).  Copies every layer's K and V block. */
int orc_copy_blocks(void* k_base, void* v_base, int64_t layer_stride_bytes, int n_layers,
                    int64_t block_bytes, int num_blocks, const int32_t* pairs, int n_pairs) {
    int bad = 0;
    for (int p = 0; p < n_pairs; ++p) {
        const int32_t src = pairs[2 * p], dst = pairs[2 * p + 1];
        if (src < 0 || dst < 0 || src >= num_blocks || dst >= num_blocks) { bad = 1; continue; }
        for (int l = 0; l < n_layers; ++l) {
            char* kb = (char*)k_base + l * layer_stride_bytes;
            char* vb = (char*)v_base + l * layer_stride_bytes;
            memcpy(kb + dst * block_bytes, kb + src * block_bytes, block_bytes);
            memcpy(vb + dst * block_bytes, vb + src * block_bytes, block_bytes);
        }
    }
    return bad ? -1 : 0;
}

/* dot product with eight partial sums (a fixed, vectorisable order) */
static inline float dot_f32(const float* a, const float* b, int n) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    int d = 0;
    for (; d + 8 <= n; d += 8)
        for (int u = 0; u < 8; ++u) acc[u] += a[d + u] * b[d + u];
    float s = ((acc[0] + acc[1]) + (acc[2] + acc[3])) + ((acc[4] + acc[5]) + (acc[6] + acc[7]));
    for (; d < n; ++d) s += a[d] * b[d];
    return s;
}
static inline double dot_f64(const float* a, const float* b, int n) {
    double s = 0.0;
    for (int d = 0; d < n; ++d) s += (double)a[d] * (double)b[d];
    return s;
}

/*
 * Unified decode / chunked-prefill attention.  Sequence s owns query rows
 * [query_start_loc[s], query_start_loc[s+1]) and attends over
 * total_s = num_prior[s] + n_new_s keys read through its block table.
 * Returns 0, or -1 when a table entry is outside the pool (that sequence's
 * output is left untouched).
 */
int orc_paged_attention(void* out, const void* q, const void* k_pool, const void* v_pool,
                        const int32_t* block_tables, int64_t bt_stride,
                        const int32_t* query_start_loc, const int32_t* num_prior, int n_seqs,
                        int n_q_heads, int n_kv_heads, int head_dim, int block_size, int num_blocks,
                        float scale, int dtype, int n_threads) {
    const int G = n_q_heads / n_kv_heads;
    const int D = head_dim;
    const int64_t n_tasks = (int64_t)n_seqs * n_q_heads;
    int bad = 0;
#ifdef _OPENMP
    if (n_threads <= 0) n_threads = omp_get_max_threads();
#pragma omp parallel num_threads(n_threads) reduction(| : bad)
#endif
    {
        float* kbuf = NULL; float* vbuf = NULL; float* sc = NULL; float* qv = NULL; double* accd = NULL;
        int64_t cap = 0;
#ifdef _OPENMP
#pragma omp for schedule(dynamic, 1)
#endif
        for (int64_t task = 0; task < n_tasks; ++task) {
            const int s = (int)(task / n_q_heads), h = (int)(task % n_q_heads), g = h / G;
            const int q0 = query_start_loc[s], n_new = query_start_loc[s + 1] - q0;
            if (n_new <= 0) continue;
            const int64_t total = (int64_t)num_prior[s] + n_new;
            const int64_t used = (total + block_size - 1) / block_size;
            if (total > cap) {
                cap = total;
                kbuf = (float*)realloc(kbuf, sizeof(float) * cap * D);
                vbuf = (float*)realloc(vbuf, sizeof(float) * cap * D);
                sc = (float*)realloc(sc, sizeof(float) * cap);
                qv = (float*)realloc(qv, sizeof(float) * D);
                accd = (double*)realloc(accd, sizeof(double) * D);
            }
            /* gather: k = k_pool[table[:used]].reshape(used*bs, ...)[:total] (kv head g) */
            int ok = 1;
            for (int64_t b = 0; b < used && ok; ++b) {
                const int32_t blk = block_tables[s * bt_stride + b];
                if (blk < 0 || blk >= num_blocks) { ok = 0; break; }
                for (int o = 0; o < block_size; ++o) {
                    const int64_t j = b * block_size + o;
                    if (j >= total) break;
                    const int64_t src = (((int64_t)blk * block_size + o) * n_kv_heads + g) * D;
                    for (int d = 0; d < D; ++d) {
                        kbuf[j * D + d] = load_el(k_pool, src + d, dtype);
                        vbuf[j * D + d] = load_el(v_pool, src + d, dtype);
                    }
                }
            }
            if (!ok) { bad = 1; continue; }
            for (int i = 0; i < n_new; ++i) {
                const int64_t qrow = ((int64_t)(q0 + i) * n_q_heads + h) * D;
                for (int d = 0; d < D; ++d) qv[d] = load_el(q, qrow + d, dtype);
                /* num_new > 1 masks kv_idx > num_prior + i; num_new == 1 masks nothing
                   (and then limit == total anyway). */
                const int64_t limit = (n_new > 1) ? (int64_t)num_prior[s] + i + 1 : total;
                float m = -INFINITY;
                for (int64_t j = 0; j < limit; ++j) {
                    float x;
                    if (dtype == ORC_F32) x = (float)(dot_f64(qv, kbuf + j * D, D) * (double)scale);
                    else x = round_dt(round_dt(dot_f32(qv, kbuf + j * D, D), dtype) * scale, dtype);
                    sc[j] = x;
                    if (x > m) m = x;
                }
                float sum = 0.f;
                for (int64_t j = 0; j < limit; ++j) { sc[j] = expf(sc[j] - m); sum += sc[j]; }
                const float inv = 1.f / sum;
                for (int64_t j = 0; j < limit; ++j) sc[j] = round_dt(sc[j] * inv, dtype);
                for (int d = 0; d < D; ++d) accd[d] = 0.0;
                if (dtype == ORC_F32) {
                    for (int64_t j = 0; j < limit; ++j)
                        for (int d = 0; d < D; ++d) accd[d] += (double)sc[j] * (double)vbuf[j * D + d];
                    for (int d = 0; d < D; ++d) store_el(out, qrow + d, (float)accd[d], dtype);
                } else {
                    float* acc = qv; /* reuse: q row no longer needed */
                    for (int d = 0; d < D; ++d) acc[d] = 0.f;
                    for (int64_t j = 0; j < limit; ++j) {
                        const float p = sc[j];
                        const float* vr = vbuf + j * D;
                        for (int d = 0; d < D; ++d) acc[d] += p * vr[d];
                    }
                    for (int d = 0; d < D; ++d) store_el(out, qrow + d, acc[d], dtype);
                }
            }
        }
        free(kbuf); free(vbuf); free(sc); free(qv); free(accd);
    }
    return bad ? -1 : 0;
}
