/*
 * asu_oracle.c -- CPU restatement of the resolver hot path (TEST INFRASTRUCTURE ONLY).
 *
 * Used by tests/ as a fast checker at large sizes and by bench.py as the timed CPU
 * baseline (its cpu_baseline leg and its --impl reference arm).  Never linked into or
 * called by the product library.  Parity: tests/test_oracle_c.py checks every function
 * here against oracle/asu_oracle.py, which is pinned to the reference's own outputs.
 *
 *  lru_*      LRUManagedCache, simu/kv_cache_eviction_sim.py:99-150 -- an OrderedDict is
 *             a doubly linked list over slots (LRU at the head) plus a key -> slot map;
 *             prepare_free_slots pops the head, resolve_query moves hits to the tail and
 *             pops the free list (a stack) for misses.  One pool per request.
 *  ops_*      ops/scripts/asu_hbm_index_common.py:119-139 (lookup) and :185-214 (maintain).
 *  gather     simu/hbm_lookup_update/scripts/test_lookup_update.py:75-78.
 *  swap-in    memcpy of each installed row from the host row pool to the slot pool.
 *
 * Multi-threading: requests are independent, so lru_step_all() splits the request rows
 * over pthreads (each thread runs the serial algorithm on its rows).
 */
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define NOT_FOUND (-1)

/* ------------------------------------------------------------------ exact LRU pool */

typedef struct {
    int32_t slots, target, key_space;
    int32_t* t2s;    /* [key_space] key -> slot, -1 absent */
    int32_t* s2t;    /* [slots] slot -> key */
    int32_t* prev;   /* linked list over resident slots, LRU at head */
    int32_t* next;
    int32_t head, tail, resident;
    int32_t* free_stack; /* [slots], top = free_stack[free_count - 1] */
    int32_t free_count;
} lru_pool;

lru_pool* lru_create(int32_t slots, int32_t target, int32_t key_space) {
    lru_pool* p = (lru_pool*)calloc(1, sizeof(lru_pool));
    if (!p) return NULL;
    p->slots = slots;
    p->target = target < slots ? target : slots;
    p->key_space = key_space;
    p->t2s = (int32_t*)malloc(sizeof(int32_t) * (size_t)key_space);
    p->s2t = (int32_t*)malloc(sizeof(int32_t) * (size_t)slots);
    p->prev = (int32_t*)malloc(sizeof(int32_t) * (size_t)slots);
    p->next = (int32_t*)malloc(sizeof(int32_t) * (size_t)slots);
    p->free_stack = (int32_t*)malloc(sizeof(int32_t) * (size_t)slots);
    if (!p->t2s || !p->s2t || !p->prev || !p->next || !p->free_stack) return NULL;
    for (int32_t k = 0; k < key_space; ++k) p->t2s[k] = NOT_FOUND;
    for (int32_t s = 0; s < slots; ++s) {
        p->s2t[s] = NOT_FOUND;
        p->free_stack[s] = slots - 1 - s; /* list(range(S-1, -1, -1)), :109 */
    }
    p->free_count = slots;
    p->head = p->tail = NOT_FOUND;
    p->resident = 0;
    return p;
}

void lru_destroy(lru_pool* p) {
    if (!p) return;
    free(p->t2s);
    free(p->s2t);
    free(p->prev);
    free(p->next);
    free(p->free_stack);
    free(p);
}

static void list_unlink(lru_pool* p, int32_t s) {
    int32_t a = p->prev[s], b = p->next[s];
    if (a != NOT_FOUND) p->next[a] = b; else p->head = b;
    if (b != NOT_FOUND) p->prev[b] = a; else p->tail = a;
}

static void list_append(lru_pool* p, int32_t s) {
    p->prev[s] = p->tail;
    p->next[s] = NOT_FOUND;
    if (p->tail != NOT_FOUND) p->next[p->tail] = s; else p->head = s;
    p->tail = s;
}

/* One step: prepare_free_slots then resolve_query.  Returns the number of evictions. */
int32_t lru_step(lru_pool* p, const int32_t* keys, int32_t q, int32_t* slot_out, uint8_t* hit, uint8_t* install,
                 int32_t* evicted, int64_t* stats /* hits, misses, installs, shortages, evictions (+=) */) {
    int32_t e = 0;
    while (p->free_count < p->target && p->resident > 0) { /* :127-130 */
        int32_t s = p->head;
        list_unlink(p, s);
        p->resident--;
        int32_t key = p->s2t[s];
        p->t2s[key] = NOT_FOUND;
        p->s2t[s] = NOT_FOUND;
        p->free_stack[p->free_count++] = s;
        if (evicted) evicted[e] = key;
        e++;
    }
    int64_t h = 0, m = 0, ins = 0, sh = 0;
    for (int32_t i = 0; i < q; ++i) { /* :137-148 */
        int32_t key = keys[i];
        int32_t s = NOT_FOUND;
        uint8_t is_hit = 0, is_inst = 0;
        if (key >= 0 && key < p->key_space) {
            s = p->t2s[key];
            if (s != NOT_FOUND) {
                is_hit = 1;
                h++;
                list_unlink(p, s);
                list_append(p, s);
            } else {
                m++;
                if (p->free_count > 0) {
                    s = p->free_stack[--p->free_count];
                    p->t2s[key] = s;
                    p->s2t[s] = key;
                    list_append(p, s);
                    p->resident++;
                    is_inst = 1;
                    ins++;
                } else {
                    sh++;
                }
            }
        }
        if (slot_out) slot_out[i] = s;
        if (hit) hit[i] = is_hit;
        if (install) install[i] = is_inst;
    }
    if (stats) {
        stats[0] += h;
        stats[1] += m;
        stats[2] += ins;
        stats[3] += sh;
        stats[4] += e;
    }
    return e;
}

/* State in the GPU layout (first resident entries of order are resident slots, LRU first). */
void lru_export(const lru_pool* p, int32_t* t2s, int32_t* s2t, int32_t* order, int32_t* free_stack,
                int32_t* free_count) {
    memcpy(t2s, p->t2s, sizeof(int32_t) * (size_t)p->key_space);
    memcpy(s2t, p->s2t, sizeof(int32_t) * (size_t)p->slots);
    int32_t i = 0;
    for (int32_t s = p->head; s != NOT_FOUND; s = p->next[s]) order[i++] = s;
    for (; i < p->slots; ++i) order[i] = NOT_FOUND;
    memcpy(free_stack, p->free_stack, sizeof(int32_t) * (size_t)p->free_count);
    for (int32_t j = p->free_count; j < p->slots; ++j) free_stack[j] = NOT_FOUND;
    *free_count = p->free_count;
}

/* ---- many requests, many threads: one step for every pool, plus the swap-in copy ---- */

typedef struct {
    lru_pool** pools;
    int32_t r0, r1, q;
    const int32_t* keys;      /* [R, q] */
    int32_t* slot_out;        /* [R, q] (nullable) */
    uint8_t* hit;             /* [R, q] */
    uint8_t* install;         /* [R, q] */
    int32_t* evicted;         /* [R, ev_stride] */
    int32_t ev_stride;
    int32_t* evicted_n;       /* [R] */
    int64_t* stats;           /* [R, 5] */
    /* swap-in (all nullable) */
    const uint8_t* host_pool; /* [pool_rows, row_bytes] */
    int64_t pool_rows, row_bytes;
    const int32_t* record;    /* [R, key_space] */
    int64_t key_space;
    uint8_t* slot_pool;       /* [R, slots, row_bytes] */
    int32_t slots;
} step_job;

static void* step_worker(void* arg) {
    step_job* j = (step_job*)arg;
    int32_t* tmp_slot = (int32_t*)malloc(sizeof(int32_t) * (size_t)j->q);
    uint8_t* tmp_inst = (uint8_t*)malloc((size_t)j->q);
    for (int32_t r = j->r0; r < j->r1; ++r) {
        const int64_t o = (int64_t)r * j->q;
        int32_t* so = j->slot_out ? j->slot_out + o : tmp_slot;
        uint8_t* in = j->install ? j->install + o : tmp_inst;
        int32_t n = lru_step(j->pools[r], j->keys + o, j->q, so, j->hit ? j->hit + o : NULL, in,
                             j->evicted ? j->evicted + (int64_t)r * j->ev_stride : NULL,
                             j->stats ? j->stats + (int64_t)r * 5 : NULL);
        if (j->evicted_n) j->evicted_n[r] = n;
        if (j->host_pool && j->slot_pool) {
            for (int32_t i = 0; i < j->q; ++i) {
                if (!in[i]) continue;
                int64_t row = j->record[(int64_t)r * j->key_space + j->keys[o + i]];
                memcpy(j->slot_pool + ((int64_t)r * j->slots + so[i]) * j->row_bytes,
                       j->host_pool + row * j->row_bytes, (size_t)j->row_bytes);
            }
        }
    }
    free(tmp_slot);
    free(tmp_inst);
    return NULL;
}

int lru_step_all(lru_pool** pools, int32_t req_num, int32_t q, const int32_t* keys, int32_t* slot_out, uint8_t* hit,
                 uint8_t* install, int32_t* evicted, int32_t ev_stride, int32_t* evicted_n, int64_t* stats,
                 const uint8_t* host_pool, int64_t pool_rows, int64_t row_bytes, const int32_t* record,
                 int64_t key_space, uint8_t* slot_pool, int32_t slots, int32_t nthreads) {
    if (nthreads < 1) nthreads = 1;
    if (nthreads > req_num) nthreads = req_num;
    if (nthreads > 256) nthreads = 256;
    pthread_t th[256];
    step_job jobs[256];
    for (int32_t t = 0; t < nthreads; ++t) {
        step_job* j = &jobs[t];
        j->pools = pools;
        j->r0 = (int32_t)((int64_t)req_num * t / nthreads);
        j->r1 = (int32_t)((int64_t)req_num * (t + 1) / nthreads);
        j->q = q;
        j->keys = keys;
        j->slot_out = slot_out;
        j->hit = hit;
        j->install = install;
        j->evicted = evicted;
        j->ev_stride = ev_stride;
        j->evicted_n = evicted_n;
        j->stats = stats;
        j->host_pool = host_pool;
        j->pool_rows = pool_rows;
        j->row_bytes = row_bytes;
        j->record = record;
        j->key_space = key_space;
        j->slot_pool = slot_pool;
        j->slots = slots;
        if (t > 0) pthread_create(&th[t], NULL, step_worker, j);
    }
    step_worker(&jobs[0]);
    for (int32_t t = 1; t < nthreads; ++t) pthread_join(th[t], NULL);
    return 0;
}

/* ------------------------------------------------------------------ ops contract */

void ops_lookup(int32_t* index, int32_t* s2i, const int32_t* free_slots, int32_t* free_head, const int32_t* query,
                int32_t* slot_out, int32_t req_num, int32_t index_size, int32_t slot_count, int32_t free_count,
                int32_t query_count) {
    for (int32_t r = 0; r < req_num; ++r) {
        int32_t* ir = index + (int64_t)r * index_size;
        int32_t head = free_head[r];
        for (int32_t i = 0; i < query_count; ++i) {
            int32_t key = query[(int64_t)r * query_count + i];
            int32_t s = ir[key];
            if (s == NOT_FOUND) {
                s = free_slots[(int64_t)r * free_count + head];
                head++;
                ir[key] = s;
                s2i[(int64_t)r * slot_count + s] = key;
            }
            slot_out[(int64_t)r * query_count + i] = s;
        }
        free_head[r] = head;
    }
}

static uint32_t hash32(uint32_t x) {
    x ^= x >> 16;
    x *= 0x7feb352dU;
    x ^= x >> 15;
    x *= 0x846ca68bU;
    x ^= x >> 16;
    return x;
}

/* Returns 0, or -1 when a row has fewer evictable slots than free_head (the reference
 * would loop forever; here the row is left after one full ring pass). */
int ops_maintain(int32_t* index, int32_t* s2i, int32_t* free_slots, int32_t* free_head, const int32_t* lq,
                 int32_t req_num, uint32_t seed, int32_t index_size, int32_t slot_count, int32_t free_count,
                 int32_t query_count) {
    int rc = 0;
    uint8_t* prot = (uint8_t*)malloc((size_t)slot_count);
    for (int32_t r = 0; r < req_num; ++r) {
        int32_t head = free_head[r];
        if (head <= 0) continue;
        memset(prot, 0, (size_t)slot_count);
        for (int32_t i = 0; i < query_count; ++i) {
            int32_t s = lq[(int64_t)r * query_count + i];
            if (s >= 0 && s < slot_count) prot[s] = 1;
        }
        int32_t* sr = s2i + (int64_t)r * slot_count;
        uint32_t slot = hash32(seed ^ (uint32_t)r) % (uint32_t)slot_count;
        for (int32_t n = 0; n < slot_count && head > 0; ++n) {
            int32_t key = sr[slot];
            if (key != NOT_FOUND && !prot[slot]) {
                sr[slot] = NOT_FOUND;
                index[(int64_t)r * index_size + key] = NOT_FOUND;
                head--;
                free_slots[(int64_t)r * free_count + head] = (int32_t)slot;
            }
            if (++slot == (uint32_t)slot_count) slot = 0;
        }
        if (head > 0) rc = -1;
        free_head[r] = head;
    }
    free(prot);
    return rc;
}

/* ------------------------------------------------------------------ gather */

void gather_lookup(const int32_t* table, int32_t index_size, const int32_t* query, int32_t qlen, int32_t* out,
                   uint8_t* hit, int32_t req_num) {
    for (int32_t r = 0; r < req_num; ++r)
        for (int32_t i = 0; i < qlen; ++i) {
            int32_t v = table[(int64_t)r * index_size + query[(int64_t)r * qlen + i]];
            out[(int64_t)r * qlen + i] = v;
            if (hit) hit[(int64_t)r * qlen + i] = v != NOT_FOUND;
        }
}
