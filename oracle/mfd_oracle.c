/*
 * mfd_oracle.c -- CPU restatement of the MFD verify-step integer/index algorithms.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker the parity tests, smoke() and the
 * cpu_baseline leg of bench.py compare the CUDA kernels against.  Nothing in the product
 * package (mfd_b200/) links, loads or calls it.
 *
 * What it restates (reference = hhhhhhy5/multi-future-drafting):
 *   - oracle_build_single   : single-mode best-first heap with the rank-tuple tie-break
 *                             (inference/hf/tree_build_ext.py:31-46, 118-156;
 *                              inference/hf/ddtree.py:161-192)
 *   - oracle_build_mixture  : K-mode mixture heap, float32 key -(float(logw)+prior),
 *                             ties by mode, parent, depth, rank, logw; dedup by (parent, token)
 *                             (inference/hf/tree_build_ext.py:48-62, 158-203;
 *                              inference/hf/ddtree.py:259-293)
 *   - oracle_build_trees    : the batched SGLang layout tree[bs,3,B+1] + counts with the tail
 *                             convention tokens 0 / depths 0 / parents -1
 *                             (sglang-v0.5.22-mfd.patch lines 1375-1407)
 *   - oracle_visibility     : ancestor-or-self matrix (inference/hf/tree_build_ext.py:92-114)
 *   - oracle_follow         : the verified-path walk (inference/hf/tree_build_ext.py:70-83,
 *                             inference/hf/ddtree.py:368-382; SGLang _ddtree_follow_kernel,
 *                             patch lines 1706-1766, which walks at most L-1 edges)
 *   - oracle_sample_rows    : this build's seeded, reproducible sampling rule (the reference
 *                             samples with torch.multinomial, hf/model/utils.py:28-35, which is
 *                             not reproducible, so parity of the sample itself is unpinned): an
 *                             inverse-CDF sample of softmax(x / T) whose every sum has a fixed
 *                             order (see sample_row below), so the CUDA kernel returns the same
 *                             token bit for bit.
 *   - oracle_argmax_rows    : torch.argmax semantics on bf16 rows (first index of the maximum).
 *
 * Build: gcc -O2 -ffp-contract=off -fPIC -shared (oracle/Makefile).  -ffp-contract=off keeps
 * every float operation an individually rounded IEEE operation, as the CUDA kernels write them.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------ child map (dedup) */

typedef struct {
    int64_t* keys;   /* (parent << 32) | (uint32)token, -1 = empty */
    int64_t* vals;
    int64_t cap;
} cmap;

static void cmap_init(cmap* m, int64_t want) {
    int64_t cap = 64;
    while (cap < 4 * want + 8) cap <<= 1;
    m->cap = cap;
    m->keys = (int64_t*)malloc(sizeof(int64_t) * cap);
    m->vals = (int64_t*)malloc(sizeof(int64_t) * cap);
    for (int64_t i = 0; i < cap; ++i) m->keys[i] = -1;
}
static void cmap_free(cmap* m) { free(m->keys); free(m->vals); }
static uint64_t cmap_hash(int64_t k) {
    uint64_t x = (uint64_t)k;
    x ^= x >> 33; x *= 0xff51afd7ed558ccdULL; x ^= x >> 33; x *= 0xc4ceb9fe1a85ec53ULL; x ^= x >> 33;
    return x;
}
static int64_t cmap_key(int64_t parent, int64_t token) {
    return (int64_t)(((uint64_t)parent << 32) | (uint64_t)(uint32_t)token);
}
static int64_t cmap_find(const cmap* m, int64_t key) {
    uint64_t h = cmap_hash(key) & (uint64_t)(m->cap - 1);
    while (m->keys[h] != -1) {
        if (m->keys[h] == key) return m->vals[h];
        h = (h + 1) & (uint64_t)(m->cap - 1);
    }
    return -1;
}
static void cmap_put(cmap* m, int64_t key, int64_t val) {
    uint64_t h = cmap_hash(key) & (uint64_t)(m->cap - 1);
    while (m->keys[h] != -1 && m->keys[h] != key) h = (h + 1) & (uint64_t)(m->cap - 1);
    m->keys[h] = key;
    m->vals[h] = val;
}

/* ------------------------------------------------------------------ mixture heap */

typedef struct {
    float key;      /* -(float(logw) + prior[mode]) */
    int mode, parent, depth, rank;
    double logw;    /* excludes the prior */
} mix_entry;

/* a pops before b (the priority_queue's Greater comparator, read as "less") */
static int mix_before(const mix_entry* a, const mix_entry* b) {
    if (a->key != b->key) return a->key < b->key;
    if (a->mode != b->mode) return a->mode < b->mode;
    if (a->parent != b->parent) return a->parent < b->parent;
    if (a->depth != b->depth) return a->depth < b->depth;
    if (a->rank != b->rank) return a->rank < b->rank;
    return a->logw < b->logw;
}

typedef struct { mix_entry* a; int64_t n, cap; } mix_heap;

static void mh_push(mix_heap* h, mix_entry e) {
    if (h->n == h->cap) { h->cap = h->cap ? 2 * h->cap : 64; h->a = (mix_entry*)realloc(h->a, sizeof(mix_entry) * h->cap); }
    int64_t i = h->n++;
    while (i > 0) {
        int64_t p = (i - 1) / 2;
        if (!mix_before(&e, &h->a[p])) break;
        h->a[i] = h->a[p];
        i = p;
    }
    h->a[i] = e;
}
static mix_entry mh_pop(mix_heap* h) {
    mix_entry top = h->a[0];
    mix_entry last = h->a[--h->n];
    int64_t i = 0;
    for (;;) {
        int64_t c = 2 * i + 1;
        if (c >= h->n) break;
        if (c + 1 < h->n && mix_before(&h->a[c + 1], &h->a[c])) ++c;
        if (!mix_before(&h->a[c], &last)) break;
        h->a[i] = h->a[c];
        i = c;
    }
    if (h->n > 0) h->a[i] = last;
    return top;
}

/*
 * lp: [K, L, k] float32, ids: [K, L, k] int64, prior: [K] float32.
 * Writes tokens[0..n-1], depths[0..n-1] (nodes 1..n) and parents[0..n] (parents[0] = -1).
 * Returns n (<= budget); *pops receives the number of heap pops (statistics only).
 */
int64_t oracle_build_mixture(const float* lp, const int64_t* ids, const float* prior, int64_t num_modes,
                             int64_t depth_limit, int64_t topk, int64_t budget, int64_t* tokens,
                             int64_t* depths, int64_t* parents, int64_t* pops) {
#define AT(m, d, r) (((m) * depth_limit + (d)) * topk + (r))
    mix_heap h = {0, 0, 0};
    cmap cm;
    cmap_init(&cm, budget + 1);
    int64_t count = 0, npop = 0;
    parents[0] = -1;
    for (int64_t m = 0; m < num_modes; ++m) {
        double lw = (double)lp[AT(m, 0, 0)];
        mix_entry e = {-((float)lw + prior[m]), (int)m, 0, 1, 0, lw};
        mh_push(&h, e);
    }
    while (h.n > 0 && count < budget) {
        mix_entry e = mh_pop(&h);
        ++npop;
        int64_t token = ids[AT(e.mode, e.depth - 1, e.rank)];
        int64_t key = cmap_key(e.parent, token);
        int64_t current = cmap_find(&cm, key);
        if (current < 0) {
            current = count + 1;
            tokens[count] = token;
            depths[count] = e.depth;
            parents[current] = e.parent;
            cmap_put(&cm, key, current);
            ++count;
        }
        if (e.rank + 1 < topk) {
            double lw = e.logw - (double)lp[AT(e.mode, e.depth - 1, e.rank)]
                        + (double)lp[AT(e.mode, e.depth - 1, e.rank + 1)];
            mix_entry s = {-((float)lw + prior[e.mode]), e.mode, e.parent, e.depth, e.rank + 1, lw};
            mh_push(&h, s);
        }
        if (e.depth < depth_limit) {
            double lw = e.logw + (double)lp[AT(e.mode, e.depth, 0)];
            mix_entry c = {-((float)lw + prior[e.mode]), e.mode, (int)current, e.depth + 1, 0, lw};
            mh_push(&h, c);
        }
    }
    free(h.a);
    cmap_free(&cm);
    if (pops) *pops = npop;
    return count;
#undef AT
}

/* ------------------------------------------------------------------ single-mode heap */

typedef struct {
    double key;     /* -logw */
    int32_t* ranks; /* rank tuple (Python tuple tie-break) */
    int nranks;
    int parent, depth, rank;
    double logw;
} single_entry;

static int ranks_cmp(const single_entry* a, const single_entry* b) {
    int n = a->nranks < b->nranks ? a->nranks : b->nranks;
    for (int i = 0; i < n; ++i)
        if (a->ranks[i] != b->ranks[i]) return a->ranks[i] < b->ranks[i] ? -1 : 1;
    if (a->nranks != b->nranks) return a->nranks < b->nranks ? -1 : 1;
    return 0;
}
static int single_before(const single_entry* a, const single_entry* b) {
    if (a->key != b->key) return a->key < b->key;
    int c = ranks_cmp(a, b);
    if (c != 0) return c < 0;
    if (a->parent != b->parent) return a->parent < b->parent;
    if (a->depth != b->depth) return a->depth < b->depth;
    if (a->rank != b->rank) return a->rank < b->rank;
    return a->logw < b->logw;
}

typedef struct { single_entry* a; int64_t n, cap; } single_heap;

static void sh_push(single_heap* h, single_entry e) {
    if (h->n == h->cap) { h->cap = h->cap ? 2 * h->cap : 64; h->a = (single_entry*)realloc(h->a, sizeof(single_entry) * h->cap); }
    int64_t i = h->n++;
    while (i > 0) {
        int64_t p = (i - 1) / 2;
        if (!single_before(&e, &h->a[p])) break;
        h->a[i] = h->a[p];
        i = p;
    }
    h->a[i] = e;
}
static single_entry sh_pop(single_heap* h) {
    single_entry top = h->a[0];
    single_entry last = h->a[--h->n];
    int64_t i = 0;
    for (;;) {
        int64_t c = 2 * i + 1;
        if (c >= h->n) break;
        if (c + 1 < h->n && single_before(&h->a[c + 1], &h->a[c])) ++c;
        if (!single_before(&h->a[c], &last)) break;
        h->a[i] = h->a[c];
        i = c;
    }
    if (h->n > 0) h->a[i] = last;
    return top;
}

/* lp: [L, k] float32, ids: [L, k] int64.  Output convention as oracle_build_mixture. */
int64_t oracle_build_single(const float* lp, const int64_t* ids, int64_t depth_limit, int64_t topk,
                            int64_t budget, int64_t* tokens, int64_t* depths, int64_t* parents,
                            int64_t* pops) {
    single_heap h = {0, 0, 0};
    int64_t count = 0, npop = 0;
    parents[0] = -1;
    {
        single_entry e;
        e.logw = (double)lp[0];
        e.key = -e.logw;
        e.ranks = (int32_t*)malloc(sizeof(int32_t));
        e.ranks[0] = 0;
        e.nranks = 1;
        e.parent = 0; e.depth = 1; e.rank = 0;
        sh_push(&h, e);
    }
    while (h.n > 0 && count < budget) {
        single_entry e = sh_pop(&h);
        ++npop;
        int64_t token = ids[(e.depth - 1) * topk + e.rank];
        int64_t current = count + 1;
        tokens[count] = token;
        depths[count] = e.depth;
        parents[current] = e.parent;
        ++count;
        if (e.rank + 1 < topk) {
            single_entry s;
            s.nranks = e.nranks;
            s.ranks = (int32_t*)malloc(sizeof(int32_t) * s.nranks);
            memcpy(s.ranks, e.ranks, sizeof(int32_t) * s.nranks);
            s.ranks[s.nranks - 1] = e.rank + 1;
            s.logw = e.logw - (double)lp[(e.depth - 1) * topk + e.rank] + (double)lp[(e.depth - 1) * topk + e.rank + 1];
            s.key = -s.logw;
            s.parent = e.parent; s.depth = e.depth; s.rank = e.rank + 1;
            sh_push(&h, s);
        }
        if (e.depth < depth_limit) {
            single_entry c;
            c.nranks = e.nranks + 1;
            c.ranks = (int32_t*)malloc(sizeof(int32_t) * c.nranks);
            memcpy(c.ranks, e.ranks, sizeof(int32_t) * e.nranks);
            c.ranks[e.nranks] = 0;
            c.logw = e.logw + (double)lp[e.depth * topk];
            c.key = -c.logw;
            c.parent = (int)current; c.depth = e.depth + 1; c.rank = 0;
            sh_push(&h, c);
        }
        free(e.ranks);
    }
    for (int64_t i = 0; i < h.n; ++i) free(h.a[i].ranks);
    free(h.a);
    if (pops) *pops = npop;
    return count;
}

/* ------------------------------------------------------------------ batched SGLang layout */

/*
 * lp: [bs, K, L, k] float32, ids: [bs, K, L, k] int32, prior: [bs, K].
 * tree: [bs, 3, budget+1] int64 (tokens, depths, parents), counts: [bs] int64.
 * K == 1 uses the single-mode heap, as the SGLang builder does.
 */
void oracle_build_trees(const float* lp, const int32_t* ids32, const float* prior, int64_t bs, int64_t num_modes,
                        int64_t depth_limit, int64_t topk, int64_t budget, int64_t* tree, int64_t* counts) {
    const int64_t width = budget + 1, per = num_modes * depth_limit * topk;
    int64_t* ids = (int64_t*)malloc(sizeof(int64_t) * (per > 0 ? per : 1));
    int64_t* tok = (int64_t*)malloc(sizeof(int64_t) * (budget > 0 ? budget : 1));
    int64_t* dep = (int64_t*)malloc(sizeof(int64_t) * (budget > 0 ? budget : 1));
    for (int64_t b = 0; b < bs; ++b) {
        for (int64_t i = 0; i < per; ++i) ids[i] = ids32[b * per + i];
        int64_t* t = tree + b * 3 * width;
        int64_t* d = t + width;
        int64_t* p = d + width;
        int64_t n;
        if (num_modes == 1)
            n = oracle_build_single(lp + b * per, ids, depth_limit, topk, budget, tok, dep, p, 0);
        else
            n = oracle_build_mixture(lp + b * per, ids, prior + b * num_modes, num_modes, depth_limit, topk, budget,
                                     tok, dep, p, 0);
        t[0] = 0;
        d[0] = 0;
        for (int64_t i = 0; i < n; ++i) { t[i + 1] = tok[i]; d[i + 1] = dep[i]; }
        for (int64_t i = n + 1; i < width; ++i) { t[i] = 0; d[i] = 0; p[i] = -1; }
        counts[b] = n;
    }
    free(ids); free(tok); free(dep);
}

/* ------------------------------------------------------------------ visibility and walk */

/* parents [m] (parents[i] < i; -1 marks a root, as node 0 of a draft tree or any node of a forest hanging off
 * the committed state) -> vis [m, m] uint8, row i = ancestors of i and i. */
void oracle_visibility(const int64_t* parents, int64_t m, uint8_t* vis) {
    memset(vis, 0, (size_t)(m * m));
    for (int64_t i = 0; i < m; ++i) {
        if (parents[i] >= 0 && parents[i] < i) memcpy(vis + i * m, vis + parents[i] * m, (size_t)i);
        vis[i * m + i] = 1;
    }
}

/*
 * Walk node 0 -> child whose token equals post[current] while one exists, at most max_steps edges
 * (max_steps < 0: unbounded, as the HF walk).  tokens[i] is node i's token (tokens[0] unused),
 * parents[i] its parent.  accepted[] receives the node indices (accepted[0] = 0); returns the count
 * and writes the bonus (post[last]) to *bonus.  Ties between children cannot occur: a parent's
 * children carry distinct tokens.
 */
int64_t oracle_follow(const int64_t* tokens, const int64_t* parents, int64_t m, const int64_t* post,
                      int64_t max_steps, int64_t* accepted, int64_t* bonus) {
    int64_t n = 0, cur = 0;
    accepted[n++] = 0;
    int64_t next = post[0];
    for (;;) {
        if (max_steps >= 0 && n - 1 >= max_steps) break;
        int64_t found = -1;
        for (int64_t i = 1; i < m; ++i)
            if (parents[i] == cur && tokens[i] == next) { found = i; break; }
        if (found < 0) break;
        cur = found;
        accepted[n++] = cur;
        next = post[cur];
    }
    *bonus = next;
    return n;
}

/* ------------------------------------------------------------------ sampling rule */

static float bf16_to_f32(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/*
 * exp(y) for y <= 0 in float32 by Cody-Waite range reduction (W. J. Cody and W. Waite,
 * "Software Manual for the Elementary Functions", 1980: ln 2 split as 0.693359375 - 2.12194440e-4)
 * and the degree-5 polynomial 1 + c1 r + ... + c5 r^5 of exp on |r| <= ln2/2 (constant term fixed at 1;
 * fitted for the least maximum relative error, 9.2e-8, by Lawson's iteratively reweighted least squares on
 * 40001 points) evaluated by Horner's rule with fmaf.
 * Every step is a single correctly rounded IEEE operation, so the CUDA kernel, which performs the
 * same operations with __fmaf_rn / __fmul_rn / __fadd_rn, returns the same bits.
 */
static float mfd_exp32(float y) {
    if (!(y > -87.0f)) return 0.0f;               /* also maps -inf and NaN to 0 */
    float n = nearbyintf(y * 1.44269504088896341f); /* round half to even, as __float2int_rn */
    float r = fmaf(n, -0.693359375f, y);
    r = fmaf(n, 2.12194440e-4f, r);
    float p = 0.008290256f;
    p = fmaf(p, r, 0.041897807f);
    p = fmaf(p, r, 0.16667636f);
    p = fmaf(p, r, 0.4999915f);
    p = fmaf(p, r, 0.9999997f);
    p = fmaf(p, r, 1.0f);
    /* scale by 2^n by adding n to the exponent field: y > -87 gives n >= -126, and n = -126 only
       when r > 0.34, i.e. p > 1, so the result stays a normal number */
    int ni = (int)n;
    uint32_t bits;
    memcpy(&bits, &p, 4);
    bits += (uint32_t)ni << 23;
    memcpy(&p, &bits, 4);
    return p;
}

float oracle_exp32(float y) { return mfd_exp32(y); }

/*
 * The sampling rule, one row x[0, V) of bf16 logits, c = 1/T (float32), u in [0, 1):
 *   blocks      b = 0 .. nb-1 of 256 logits (positions past V count as -inf); lane l of a block holds its
 *               logits 8l .. 8l+7.
 *   block max   M_b (float32 maximum; -inf for a block of -inf).
 *   weights     e_i = exp32((x_i - M_b) * c) in float32 (0 when M_b = -inf).
 *   block sum   s_l = e_{8l} + ... + e_{8l+7} added left to right in float32, then the 32 lane sums by the
 *               butterfly v_l <- v_l + v_{l xor o} for o = 16, 8, 4, 2, 1; S_b = v_0.
 *   row max     m = max_b M_b;  block weight w_b = (double)S_b * (double)exp32((M_b - m) * c) (0 for M_b = -inf).
 *   runs        run L = blocks [L p, L p + p), p = ceil(nb / 32), L = 0 .. 31; R_L = sum of its w_b left to right
 *               in double from 0.
 *   total       P_0 = 0, P_{L+1} = P_L + R_L in double; Z = P_32; Z = 0 (every logit -inf): token V - 1.
 *   target      t = u Z.
 *   run         L* = first L with P_{L+1} > t; t1 = t - P_{L*}.
 *   block       Q = 0; for b in run L*: Q' = Q + w_b; first b with Q' > t1 is b*, t2 = t1 - Q.
 *   lane        in b*, c_l = sum over its 8 logits of (double)e_i * sc (sc = exp32((M_b* - m) * c)) left to right
 *               from 0; B_0 = 0, B_{l+1} = B_l + c_l; l* = first l with B_{l+1} > t2; t3 = t2 - B_{l*}.
 *   logit       a = 0; for the 8 logits j of lane l*: a' = a + (double)e_j * sc; first j with a' > t3 and a
 *               positive weight is the token.
 *   Where rounding leaves a level without a crossing, the token is the last logit of positive weight in that
 *   level's range (the run, the block, the lane).
 * Every block is reduced independently (one pass over the logits on the GPU: block maximum, then weights), and
 * every later sum has the order written above, so the kernel and this restatement agree bit for bit.
 */
static float row_x(const uint16_t* x, int64_t V, int64_t i) { return i < V ? bf16_to_f32(x[i]) : -INFINITY; }

static int64_t last_positive(const uint16_t* x, int64_t V, int64_t lo, int64_t hi, const float* M, float inv_temp) {
    /* the last logit of positive weight in [lo, hi), or -1 */
    for (int64_t i = (hi < V ? hi : V) - 1; i >= lo; --i) {
        const float mb = M[i / 256];
        if (mb == -INFINITY) continue;
        if (mfd_exp32((row_x(x, V, i) - mb) * inv_temp) > 0.0f) return i;
    }
    return -1;
}

static int64_t sample_row(const uint16_t* x, int64_t V, float inv_temp, double u, float* M, float* S) {
    const int64_t nb = (V + 255) / 256;
    for (int64_t b = 0; b < nb; ++b) {
        float mb = -INFINITY;
        for (int64_t i = 256 * b; i < 256 * b + 256; ++i) { const float v = row_x(x, V, i); if (v > mb) mb = v; }
        float lane[32], tmp[32];
        for (int l = 0; l < 32; ++l) {
            float s = 0.0f;
            for (int j = 0; j < 8; ++j) {
                const float v = row_x(x, V, 256 * b + 8 * l + j);
                const float e = mb == -INFINITY ? 0.0f : mfd_exp32((v - mb) * inv_temp);
                s = s + e;
            }
            lane[l] = s;
        }
        for (int o = 16; o >= 1; o >>= 1) {
            for (int l = 0; l < 32; ++l) tmp[l] = lane[l] + lane[l ^ o];
            memcpy(lane, tmp, sizeof(lane));
        }
        M[b] = mb;
        S[b] = lane[0];
    }
    float m = -INFINITY;
    for (int64_t b = 0; b < nb; ++b) if (M[b] > m) m = M[b];
    const int64_t per = (nb + 31) / 32;
#define W_OF(b) (M[b] == -INFINITY ? 0.0 : (double)S[b] * (double)mfd_exp32((M[b] - m) * inv_temp))
    double R[32], P[33];
    for (int L = 0; L < 32; ++L) {
        double acc = 0.0;
        for (int64_t b = L * per; b < (L + 1) * per && b < nb; ++b) acc = acc + W_OF(b);
        R[L] = acc;
    }
    P[0] = 0.0;
    for (int L = 0; L < 32; ++L) P[L + 1] = P[L] + R[L];
    const double Z = P[32];
    if (!(Z > 0.0)) return V - 1;
    const double t = u * Z;
    int Ls = -1;
    for (int L = 0; L < 32; ++L) if (P[L + 1] > t) { Ls = L; break; }
    if (Ls < 0) { const int64_t f = last_positive(x, V, 0, 256 * nb, M, inv_temp); return f < 0 ? V - 1 : f; }
    const double t1 = t - P[Ls];
    int64_t bs = -1;
    double t2 = 0.0;
    {
        double Q = 0.0;
        for (int64_t b = Ls * per; b < (Ls + 1) * per && b < nb; ++b) {
            const double Qn = Q + W_OF(b);
            if (Qn > t1) { bs = b; t2 = t1 - Q; break; }
            Q = Qn;
        }
    }
    if (bs < 0) {
        const int64_t f = last_positive(x, V, 256 * (Ls * per), 256 * ((Ls + 1) * per), M, inv_temp);
        return f < 0 ? V - 1 : f;
    }
    const float mb = M[bs];
    const double sc = (double)mfd_exp32((mb - m) * inv_temp);
    double B = 0.0, t3 = 0.0;
    int ls = -1;
    for (int l = 0; l < 32; ++l) {
        double cl = 0.0;
        for (int j = 0; j < 8; ++j) cl = cl + (double)mfd_exp32((row_x(x, V, 256 * bs + 8 * l + j) - mb) * inv_temp) * sc;
        const double Bn = B + cl;
        if (Bn > t2) { ls = l; t3 = t2 - B; break; }
        B = Bn;
    }
    if (ls < 0) { const int64_t f = last_positive(x, V, 256 * bs, 256 * bs + 256, M, inv_temp); return f < 0 ? V - 1 : f; }
    double a = 0.0;
    for (int j = 0; j < 8; ++j) {
        const double w = (double)mfd_exp32((row_x(x, V, 256 * bs + 8 * ls + j) - mb) * inv_temp) * sc;
        const double an = a + w;
        if (an > t3 && w > 0.0) return 256 * bs + 8 * ls + j;
        a = an;
    }
    {
        const int64_t f = last_positive(x, V, 256 * bs + 8 * ls, 256 * bs + 8 * ls + 8, M, inv_temp);
        return f < 0 ? V - 1 : f;
    }
#undef W_OF
}

/*
 * rows: [R, V] bf16 (as uint16), inv_temp: 1/T as float32, u: [R] float64 uniforms in [0, 1).
 * out: [R] int64 sampled token per row (the rule above).
 */
void oracle_sample_rows(const uint16_t* rows, int64_t R, int64_t V, float inv_temp, const double* u, int64_t* out) {
    const int64_t nb = (V + 255) / 256;
    float* M = (float*)malloc(sizeof(float) * (size_t)nb);
    float* S = (float*)malloc(sizeof(float) * (size_t)nb);
    for (int64_t r = 0; r < R; ++r) out[r] = sample_row(rows + r * V, V, inv_temp, u[r], M, S);
    free(M);
    free(S);
}

/* rows [R, V] bf16 -> first index of the row maximum (torch.argmax on finite values). */
void oracle_argmax_rows(const uint16_t* rows, int64_t R, int64_t V, int64_t* out) {
    for (int64_t r = 0; r < R; ++r) {
        const uint16_t* x = rows + r * V;
        float best = bf16_to_f32(x[0]);
        int64_t bi = 0;
        for (int64_t i = 1; i < V; ++i) {
            float v = bf16_to_f32(x[i]);
            if (v > best) { best = v; bi = i; }
        }
        out[r] = bi;
    }
}
