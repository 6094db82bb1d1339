/*
 * ORACLE - test infrastructure only.  Nothing in the product links, loads or calls this file;
 * it is the CPU reference the parity tests compare the CUDA library against.
 *
 * Plain-C restatement of
 *   (1) one POV iteration with given randomness: the reference kernel's semantics
 *       (src/povs/__cuda/lib/povs.cu:203-221 member sort, :225-278 gather at offset-wrapped
 *       rows, :282-321 gap-free slot index, :325-348 permuted write-back), with the NumPy
 *       path's member order as an option (src/povs/numpy.py:120-136);
 *   (2) the library's device randomness (Philox4x32-10 of Salmon et al., SC'11; a 12-round
 *       Feistel bijection with cycle walking for the pblock -> vblock map; per-vblock orders
 *       from sorting packed 32-bit (key | element) words), so the default GPU mode can be
 *       checked bit-exactly.
 * Written independently of the CUDA sources; Philox is pinned by the Random123 known-answer
 * vectors in the tests.
 */
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* ---------------------------------------------------------------- Philox4x32-10 */

static void ph_mulhilo(uint32_t a, uint32_t b, uint32_t* hi, uint32_t* lo)
{
    uint64_t prod = (uint64_t)a * (uint64_t)b;
    *hi = (uint32_t)(prod >> 32);
    *lo = (uint32_t)prod;
}

void oracle_philox4x32_10(const uint32_t ctr_in[4], const uint32_t key_in[2], uint32_t out[4])
{
    uint32_t c0 = ctr_in[0], c1 = ctr_in[1], c2 = ctr_in[2], c3 = ctr_in[3];
    uint32_t k0 = key_in[0], k1 = key_in[1];
    for (int round = 0; round < 10; ++round) {
        uint32_t h0, l0, h1, l1;
        ph_mulhilo(0xD2511F53u, c0, &h0, &l0);
        ph_mulhilo(0xCD9E8D57u, c2, &h1, &l1);
        uint32_t n0 = h1 ^ c1 ^ k0;
        uint32_t n1 = l1;
        uint32_t n2 = h0 ^ c3 ^ k1;
        uint32_t n3 = l0;
        c0 = n0;
        c1 = n1;
        c2 = n2;
        c3 = n3;
        k0 += 0x9E3779B9u;
        k1 += 0xBB67AE85u;
    }
    out[0] = c0;
    out[1] = c1;
    out[2] = c2;
    out[3] = c3;
}

enum { DOM_OFFSET = 1, DOM_ASSIGN = 2, DOM_PERM = 3, DOM_VSEED = 4, N_FEISTEL = 12 };

/* Randomness modes: 0 = uniform permutations; 1 = the reference CUDA path's distribution. */
enum { MODE_UNIFORM = 0, MODE_REFERENCE_CUDA = 1, MODE_REFERENCE_NUMPY = 2 };

/*
 * Mode 2 (the reference NumPy path's distribution): the permutation of a vblock of n valid rows
 * under per-vblock seed s in 1..999 is numpy.random.RandomState(s).shuffle(arange(n)), taken from a
 * table that the caller builds with NumPy itself (oracle/api.py): np_table[np_off[c] + (s-1)*n + f],
 * class c = n/P - 1 for whole members, V + (n - n_rows % P)/P with the truncated last pblock.
 */
static const int32_t* np_table = NULL;
static int64_t np_off[64];
static int np_P = 0, np_V = 0;
static int64_t np_trunc = 0;

void oracle_set_numpy_table(const int32_t* table, const int64_t* off, int P, int V, int64_t trunc)
{
    np_table = table;
    for (int i = 0; i < 2 * V && i < 64; ++i) np_off[i] = off[i];
    np_P = P;
    np_V = V;
    np_trunc = trunc;
}

static const int32_t* numpy_perm(int n, uint32_t s)
{
    const int cls = (n % np_P) == 0 ? n / np_P - 1 : np_V + (int)((n - np_trunc) / np_P);
    return np_table + np_off[cls] + (int64_t)(s - 1u) * n;
}

static void draw(uint64_t seed, uint32_t c0, uint32_t c1, uint32_t c2, uint32_t c3, uint32_t out[4])
{
    uint32_t ctr[4] = {c0, c1, c2, c3};
    uint32_t key[2] = {(uint32_t)seed, (uint32_t)(seed >> 32)};
    oracle_philox4x32_10(ctr, key, out);
}

/* ---------------------------------------------------------------- Feistel bijection */

static uint32_t mix32(uint32_t x)
{
    x ^= x >> 16;
    x *= 0x7feb352du;
    x ^= x >> 15;
    x *= 0x846ca68bu;
    x ^= x >> 16;
    return x;
}

typedef struct {
    uint32_t key[N_FEISTEL];
    uint64_t n;
    int hi_bits, lo_bits;
} bijection_t;

static void bijection_init(bijection_t* b, uint64_t seed, uint32_t iteration, uint64_t n)
{
    for (uint32_t c = 0; c < N_FEISTEL / 4; ++c) {
        uint32_t r[4];
        draw(seed, c, 0u, (uint32_t)DOM_ASSIGN << 24, iteration, r);
        for (int t = 0; t < 4; ++t) b->key[4 * c + t] = r[t];
    }
    b->n = n;
    int bits = 2;
    while (bits < 64 && ((uint64_t)1 << bits) < n) bits++;
    b->hi_bits = bits / 2;
    b->lo_bits = bits - b->hi_bits;
}

/* One pass of the network: state (hi, lo) of widths (wh, wl) -> (lo, hi ^ F(lo)) of widths (wl, wh). */
static uint64_t bijection_pass(const bijection_t* b, uint64_t x)
{
    int wh = b->hi_bits, wl = b->lo_bits;
    uint64_t hi = x >> wl, lo = x & (((uint64_t)1 << wl) - 1);
    for (int i = 0; i < N_FEISTEL; ++i) {
        uint32_t f0 = mix32((uint32_t)lo ^ b->key[i]);
        uint32_t f1 = mix32((uint32_t)(lo >> 32) ^ f0 ^ b->key[(i + 1) % N_FEISTEL]);
        uint64_t f = ((uint64_t)f1 << 32) | f0;
        uint64_t new_lo = (hi ^ f) & (((uint64_t)1 << wh) - 1);
        hi = lo;
        lo = new_lo;
        int tmp = wh;
        wh = wl;
        wl = tmp;
    }
    return (hi << wl) | lo;
}

static uint64_t bijection_apply(const bijection_t* b, uint64_t x)
{
    uint64_t y = bijection_pass(b, x);
    while (y >= b->n) y = bijection_pass(b, y);
    return y;
}

/* ---------------------------------------------------------------- iteration semantics */

typedef struct {
    int64_t id;
    int order_key_class; /* used by the given-order mode */
    int pos;
} member_t;

static int cmp_member_sorted(const void* a, const void* b)
{
    const member_t* x = (const member_t*)a;
    const member_t* y = (const member_t*)b;
    /* valid ascending, padding (id < 0) last, ties by position */
    int xv = x->id >= 0, yv = y->id >= 0;
    if (xv != yv) return xv ? -1 : 1;
    if (xv && x->id != y->id) return x->id < y->id ? -1 : 1;
    return x->pos - y->pos;
}

static int cmp_member_given(const void* a, const void* b)
{
    const member_t* x = (const member_t*)a;
    const member_t* y = (const member_t*)b;
    if (x->order_key_class != y->order_key_class) return x->order_key_class - y->order_key_class;
    return x->pos - y->pos;
}

/*
 * Orders the members of one vblock and returns the number of valid rows; starts[r] receives the
 * storage row of the first row of the r-th ordered valid member.
 */
static int order_members(const int64_t* assign_row, int V, int64_t N, int P, int64_t n_p, int64_t offset,
                         int sort_members, int64_t* starts, int* n_members)
{
    member_t m[64];
    for (int k = 0; k < V; ++k) {
        int64_t a = assign_row[k];
        m[k].id = (a >= 0 && a < n_p) ? a : -1;
        m[k].pos = k;
        if (m[k].id < 0) {
            m[k].order_key_class = 2;
        } else {
            int64_t rows = N - m[k].id * P;
            m[k].order_key_class = rows < P ? 1 : 0;
        }
    }
    qsort(m, (size_t)V, sizeof(member_t), sort_members ? cmp_member_sorted : cmp_member_given);
    int n_valid = 0, nm = 0;
    for (int r = 0; r < V; ++r) {
        if (m[r].id < 0) break;
        int64_t left = N - m[r].id * P;
        int rows = left < P ? (int)left : P;
        starts[r] = (m[r].id * P + offset) % N;
        n_valid += rows;
        nm++;
    }
    *n_members = nm;
    return n_valid;
}

static int64_t slot_to_row(const int64_t* starts, int f, int P, int64_t N)
{
    int64_t row = starts[f / P] + (f % P);
    return row >= N ? row - N : row;
}

/*
 * One iteration with given randomness.
 *   assign  [n_v][V]   member ids (padding: < 0 or >= n_p)
 *   perms   [n_v][V*P] destination slot f receives source slot perms[f]
 * Returns 0, or -1 if a permutation entry is out of range.
 */
int oracle_apply_iteration(uint8_t* data, int64_t N, int64_t R, int P, int V, int64_t offset, const int64_t* assign,
                           const int32_t* perms, int sort_members)
{
    const int64_t n_p = (N + P - 1) / P;
    const int64_t n_v = (n_p + V - 1) / V;
    const int VP = V * P;
    uint8_t* tmp = (uint8_t*)malloc((size_t)VP * (size_t)R);
    if (!tmp) return -2;
    int64_t starts[64];
    for (int64_t v = 0; v < n_v; ++v) {
        int nm = 0;
        int n_valid = order_members(assign + v * V, V, N, P, n_p, offset, sort_members, starts, &nm);
        for (int f = 0; f < n_valid; ++f) {
            int64_t row = slot_to_row(starts, f, P, N);
            memcpy(tmp + (size_t)f * R, data + row * R, (size_t)R);
        }
        const int32_t* pv = perms + v * VP;
        for (int f = 0; f < n_valid; ++f) {
            if (pv[f] < 0 || pv[f] >= n_valid) {
                free(tmp);
                return -1;
            }
        }
        for (int f = 0; f < n_valid; ++f) {
            int64_t row = slot_to_row(starts, f, P, N);
            memcpy(data + row * R, tmp + (size_t)pv[f] * R, (size_t)R);
        }
    }
    free(tmp);
    return 0;
}

/* ---------------------------------------------------------------- the library's device randomness */

/* Seed in [1, 999] of vblock v (reference-CUDA mode). */
static uint32_t vblock_seed(uint64_t seed, uint32_t iteration, uint64_t v)
{
    uint32_t w[4];
    draw(seed, 0u, (uint32_t)v, ((uint32_t)(v >> 32) & 0x00FFFFFFu) | ((uint32_t)DOM_VSEED << 24), iteration, w);
    return 1u + (uint32_t)(((uint64_t)w[0] * 999u) >> 32);
}

/* The reference kernel's single-thread shuffle of the gap-free slots (povs.cu:282-321). */
static void xorshift_fisher_yates(uint32_t r, int n_valid, int32_t* perm)
{
    for (int f = 0; f < n_valid; ++f) perm[f] = f;
    const int last = n_valid - 1;
    for (int i = 0; i <= last; ++i) {
        r ^= r << 13;
        r ^= r >> 17;
        r ^= r << 5;
        int j = i + (int)(((uint64_t)r * (uint64_t)(last - i + 1)) >> 32);
        int32_t t = perm[i];
        perm[i] = perm[j];
        perm[j] = t;
    }
}

typedef struct {
    uint64_t key;
    int32_t e;
} keyed_t;

/* Sort key of element e of a vblock of up to VP slots (the device's packed 32-bit key): the
 * element's Philox word with its low idx_bits bits replaced by e, idx_bits = log2 of the sort width
 * max(32, next power of two >= VP) (povs_kernel.cuh: PermKey, perm_sort_keys). */
static uint64_t perm_sort_key(uint32_t w, int e, int VP)
{
    int width = 32;
    while (width < VP) width <<= 1;
    const uint32_t mask = (uint32_t)width - 1u;
    return (uint64_t)((w & ~mask) | (uint32_t)e);
}

static int cmp_keyed(const void* a, const void* b)
{
    const keyed_t* x = (const keyed_t*)a;
    const keyed_t* y = (const keyed_t*)b;
    if (x->key != y->key) return x->key < y->key ? -1 : 1;
    return x->e - y->e;
}

/*
 * Randomness of iteration `iteration` for `seed`: the chosen offset, the assignment [n_v][V]
 * (padding = -1) and the permutations [n_v][V*P] (entries beyond each vblock's valid rows = -1).
 */
int oracle_device_randomness(uint64_t seed, uint32_t iteration, int64_t N, int P, int V, const int64_t* offsets,
                             int n_offsets, int64_t* out_offset, int64_t* out_assign, int32_t* out_perms, int mode)
{
    const int64_t n_p = (N + P - 1) / P;
    const int64_t n_v = (n_p + V - 1) / V;
    const int VP = V * P;
    uint32_t r[4];
    draw(seed, 0u, 0u, (uint32_t)DOM_OFFSET << 24, iteration, r);
    const uint32_t idx = (uint32_t)(((uint64_t)r[0] * (uint64_t)n_offsets) >> 32);
    const int64_t offset = offsets[idx];
    *out_offset = offset;

    bijection_t b;
    /* mode 1: the bijection covers the n_p pblocks only; slots n_p.. stay padding (last vblock). */
    bijection_init(&b, seed, iteration, mode == MODE_REFERENCE_CUDA ? (uint64_t)n_p : (uint64_t)(n_v * V));
    for (int64_t s = 0; s < n_v * V; ++s) {
        if (mode == MODE_REFERENCE_CUDA && s >= n_p) {
            out_assign[s] = -1;
            continue;
        }
        uint64_t a = bijection_apply(&b, (uint64_t)s);
        out_assign[s] = (int64_t)a < n_p ? (int64_t)a : -1;
    }

    keyed_t* keys = (keyed_t*)malloc(sizeof(keyed_t) * (size_t)VP);
    if (!keys) return -2;
    int64_t starts[64];
    for (int64_t v = 0; v < n_v; ++v) {
        int nm = 0;
        int n_valid = order_members(out_assign + v * V, V, N, P, n_p, offset, mode == MODE_REFERENCE_NUMPY ? 0 : 1,
                                    starts, &nm);
        if (mode == MODE_REFERENCE_NUMPY) {
            int32_t* pv = out_perms + v * VP;
            if (np_table == NULL || np_P != P || np_V != V || np_trunc != N % P) {
                free(keys);
                return -3;
            }
            const int32_t* src = n_valid > 0 ? numpy_perm(n_valid, vblock_seed(seed, iteration, (uint64_t)v)) : NULL;
            for (int f = 0; f < VP; ++f) pv[f] = f < n_valid ? src[f] : -1;
            continue;
        }
        if (mode == MODE_REFERENCE_CUDA) {
            int32_t* pv = out_perms + v * VP;
            xorshift_fisher_yates(vblock_seed(seed, iteration, (uint64_t)v), n_valid, pv);
            for (int f = n_valid; f < VP; ++f) pv[f] = -1;
            continue;
        }
        for (int e = 0; e < n_valid; ++e) {
            uint32_t w[4];
            draw(seed, (uint32_t)e >> 2, (uint32_t)v, ((uint32_t)((uint64_t)v >> 32) & 0x00FFFFFFu) | ((uint32_t)DOM_PERM << 24),
                 iteration, w);
            keys[e].key = perm_sort_key(w[e & 3], e, VP);
            keys[e].e = e;
        }
        qsort(keys, (size_t)n_valid, sizeof(keyed_t), cmp_keyed);
        int32_t* pv = out_perms + v * VP;
        for (int f = 0; f < VP; ++f) pv[f] = f < n_valid ? keys[f].e : -1;
    }
    free(keys);
    return 0;
}

/* Full shuffle with the library's device randomness: iterations 0..iterations-1 of `seed` in `mode`. */
int oracle_shuffle(uint8_t* data, int64_t N, int64_t R, int P, int V, const int64_t* offsets, int n_offsets,
                   int iterations, uint64_t seed, int mode)
{
    const int64_t n_p = (N + P - 1) / P;
    const int64_t n_v = (n_p + V - 1) / V;
    int64_t* assign = (int64_t*)malloc(sizeof(int64_t) * (size_t)(n_v * V));
    int32_t* perms = (int32_t*)malloc(sizeof(int32_t) * (size_t)(n_v * V * P));
    if (!assign || !perms) {
        free(assign);
        free(perms);
        return -2;
    }
    int rc = 0;
    for (int it = 0; it < iterations && rc == 0; ++it) {
        int64_t offset = 0;
        rc = oracle_device_randomness(seed, (uint32_t)it, N, P, V, offsets, n_offsets, &offset, assign, perms, mode);
        if (rc == 0) rc = oracle_apply_iteration(data, N, R, P, V, offset, assign, perms, mode == MODE_REFERENCE_NUMPY ? 0 : 1);
    }
    free(assign);
    free(perms);
    return rc;
}

/* Exposed for tests of the bijection alone. */
void oracle_assignment(uint64_t seed, uint32_t iteration, int64_t n_slots, int64_t* out)
{
    bijection_t b;
    bijection_init(&b, seed, iteration, (uint64_t)n_slots);
    for (int64_t s = 0; s < n_slots; ++s) out[s] = (int64_t)bijection_apply(&b, (uint64_t)s);
}

/* ---------------------------------------------------------------- multithreaded shuffle (CPU baseline) */

typedef struct {
    uint8_t* data;
    int64_t N, R;
    int P, V;
    uint64_t seed;
    uint32_t iteration;
    int64_t offset;
    const bijection_t* bij;
    int64_t v_begin, v_end;
    int rc;
} mt_task_t;

static void* mt_worker(void* arg)
{
    mt_task_t* t = (mt_task_t*)arg;
    const int64_t n_p = (t->N + t->P - 1) / t->P;
    const int VP = t->V * t->P;
    uint8_t* tmp = (uint8_t*)malloc((size_t)VP * (size_t)t->R);
    keyed_t* keys = (keyed_t*)malloc(sizeof(keyed_t) * (size_t)VP);
    if (!tmp || !keys) {
        t->rc = -2;
        free(tmp);
        free(keys);
        return NULL;
    }
    int64_t assign[64], starts[64];
    for (int64_t v = t->v_begin; v < t->v_end; ++v) {
        for (int k = 0; k < t->V; ++k) {
            uint64_t a = bijection_apply(t->bij, (uint64_t)(v * t->V + k));
            assign[k] = (int64_t)a < n_p ? (int64_t)a : -1;
        }
        int nm = 0;
        int n_valid = order_members(assign, t->V, t->N, t->P, n_p, t->offset, 1, starts, &nm);
        for (int e = 0; e < n_valid; ++e) {
            uint32_t w[4];
            draw(t->seed, (uint32_t)e >> 2, (uint32_t)v,
                 ((uint32_t)((uint64_t)v >> 32) & 0x00FFFFFFu) | ((uint32_t)DOM_PERM << 24), t->iteration, w);
            keys[e].key = perm_sort_key(w[e & 3], e, t->V * t->P);
            keys[e].e = e;
        }
        qsort(keys, (size_t)n_valid, sizeof(keyed_t), cmp_keyed);
        for (int f = 0; f < n_valid; ++f)
            memcpy(tmp + (size_t)f * t->R, t->data + slot_to_row(starts, f, t->P, t->N) * t->R, (size_t)t->R);
        for (int f = 0; f < n_valid; ++f)
            memcpy(t->data + slot_to_row(starts, f, t->P, t->N) * t->R, tmp + (size_t)keys[f].e * t->R, (size_t)t->R);
    }
    free(tmp);
    free(keys);
    return NULL;
}

/* Same result as oracle_shuffle, with the vblocks of each iteration split over `threads` threads. */
int oracle_shuffle_threads(uint8_t* data, int64_t N, int64_t R, int P, int V, const int64_t* offsets, int n_offsets,
                           int iterations, uint64_t seed, int threads)
{
    if (threads < 1) threads = 1;
    if (threads > 512) threads = 512;
    const int64_t n_p = (N + P - 1) / P;
    const int64_t n_v = (n_p + V - 1) / V;
    pthread_t tid[512];
    mt_task_t task[512];
    for (int it = 0; it < iterations; ++it) {
        uint32_t r[4];
        draw(seed, 0u, 0u, (uint32_t)DOM_OFFSET << 24, (uint32_t)it, r);
        const int64_t offset = offsets[(uint32_t)(((uint64_t)r[0] * (uint64_t)n_offsets) >> 32)];
        bijection_t b;
        bijection_init(&b, seed, (uint32_t)it, (uint64_t)(n_v * V));
        int started = 0;
        for (int k = 0; k < threads; ++k) {
            mt_task_t* t = &task[k];
            t->data = data;
            t->N = N;
            t->R = R;
            t->P = P;
            t->V = V;
            t->seed = seed;
            t->iteration = (uint32_t)it;
            t->offset = offset;
            t->bij = &b;
            t->v_begin = n_v * k / threads;
            t->v_end = n_v * (k + 1) / threads;
            t->rc = 0;
            if (pthread_create(&tid[k], NULL, mt_worker, t) != 0) break;
            started++;
        }
        int rc = started == threads ? 0 : -3;
        for (int k = 0; k < started; ++k) {
            pthread_join(tid[k], NULL);
            if (task[k].rc) rc = task[k].rc;
        }
        if (rc) return rc;
    }
    return 0;
}
