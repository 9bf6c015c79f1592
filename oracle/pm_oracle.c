/*
 * pm_oracle.c -- CPU restatement of PagedMoE's per-step token-selection path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product links, loads or calls this
 * file; only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg
 * do, and only as the checker.  It is written independently of the CUDA
 * sources: the two implementations agree because they follow the same
 * written definition, not because they share code.
 *
 * Parity status (see the per-function notes):
 *   - greedy argmax and equality acceptance: pinned against the reference's
 *     own code (pagedmoe/lookup_decode.py:319-373, verify_decode.py:874-922)
 *     run here on numpy-backed arrays, tests/golden/make_golden.py;
 *   - constrained-decoding mask: pinned against think_budget.py:75-109;
 *   - penalties, top-k/top-p/min-p, temperature, the categorical draw:
 *     PARITY UNPINNED.  Their arithmetic lives in mlx-lm 0.31.3
 *     (mlx_lm/sample_utils.py, pinned at reference requirements.txt:2) which is
 *     darwin-only and not part of the reference tree; these functions restate
 *     its published behaviour;
 *   - residual rejection sampling: PARITY UNPINNED (no reference
 *     implementation; restates Leviathan et al. 2023 / Chen et al. 2023).
 *
 * Numerics are defined so that a GPU can reproduce them bit for bit:
 *   - EXPF / EXP64 / LOG64 below are this project's own functions (Cody & Waite
 *     1980 range reduction, Taylor / atanh series), evaluated with explicit
 *     fused multiply-adds and nothing else, so C and CUDA give identical bits;
 *   - the row log-sum-exp is taken over fixed 1024-token tiles: per tile an
 *     exact integer sum of floor(exp(x - tile_max) * 2^52), then an fp64
 *     pairwise tree over tiles (padded to a power of two with zeros);
 *   - ranking is (processed logit descending, token index ascending).
 *
 * Build: oracle/Makefile (gcc -O2 -ffp-contract=off -shared).  Row-parallel
 * drivers call the batch functions on row ranges from several host threads.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ORC_TILE 1024
#define ORC_OK 0
#define ORC_ERR_ARG (-1)

/* ------------------------------------------------------------------------ */
/* Deterministic elementary functions                                       */
/* ------------------------------------------------------------------------ */

/* e^d in fp32 for d <= ~0.  Cody-Waite reduction d = k ln2 + r with ln2 split
 * into a 16-bit head and a tail, |r| <= ln2/2, then the degree-7 Taylor
 * polynomial of e^r by Horner with fmaf, then an exact scaling by 2^k.
 * d < -87 (or NaN) returns 0. */
float orc_expf(float d)
{
    if (!(d >= -87.0f)) return 0.0f;
    const float t = d * 0x1.715476p+0f;
    const float kf = (t + 12582912.0f) - 12582912.0f; /* round half even, |t| < 2^22 */
    float r = fmaf(-kf, 0x1.62e4p-1f, d);
    r = fmaf(-kf, 0x1.7f7d1cp-20f, r);
    float p = 0x1.a01a02p-13f;
    p = fmaf(p, r, 0x1.6c16c2p-10f);
    p = fmaf(p, r, 0x1.111112p-7f);
    p = fmaf(p, r, 0x1.555556p-5f);
    p = fmaf(p, r, 0x1.555556p-3f);
    p = fmaf(p, r, 0x1.0p-1f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    return ldexpf(p, (int)kf);
}

/* floor(e^d * 2^52) as an integer; d < -38 (or NaN / -inf) gives 0.
 * e^-38 < 2^-52, so the cut never drops a non-zero term. */
uint64_t orc_q52(float d)
{
    if (!(d >= -38.0f)) return 0;
    const float e = orc_expf(d);
    return (uint64_t)(e * 0x1p52f); /* exact product, truncating conversion */
}

/* e^d in fp64 for d <= ~0; d < -700 (or NaN) returns 0.  Cody-Waite with a
 * 42-bit head of ln2, degree-13 Taylor polynomial. */
double orc_exp64(double d)
{
    if (!(d >= -700.0)) return 0.0;
    const double kd = nearbyint(d * 0x1.71547652b82fep+0);
    double r = fma(-kd, 0x1.62e42fefa3800p-1, d);
    r = fma(-kd, 0x1.ef35793c76730p-45, r);
    double p = 0x1.6124613a86d09p-33;
    p = fma(p, r, 0x1.1eed8eff8d898p-29);
    p = fma(p, r, 0x1.ae64567f544e4p-26);
    p = fma(p, r, 0x1.27e4fb7789f5cp-22);
    p = fma(p, r, 0x1.71de3a556c734p-19);
    p = fma(p, r, 0x1.a01a01a01a01ap-16);
    p = fma(p, r, 0x1.a01a01a01a01ap-13);
    p = fma(p, r, 0x1.6c16c16c16c17p-10);
    p = fma(p, r, 0x1.1111111111111p-7);
    p = fma(p, r, 0x1.5555555555555p-5);
    p = fma(p, r, 0x1.5555555555555p-3);
    p = fma(p, r, 0x1.0p-1);
    p = fma(p, r, 1.0);
    p = fma(p, r, 1.0);
    return ldexp(p, (int)kd);
}

/* natural log in fp64 for a positive normal z.  z = f 2^e with f in
 * [sqrt(1/2), sqrt(2)); log f = 2 atanh(s), s = (f-1)/(f+1), by its odd
 * series to s^23; log z = e ln2 + log f. */
double orc_log64(double z)
{
    uint64_t b;
    memcpy(&b, &z, 8);
    int e = (int)((b >> 52) & 0x7ff) - 1023;
    b = (b & 0x000fffffffffffffULL) | 0x3ff0000000000000ULL;
    double f;
    memcpy(&f, &b, 8);
    if (f > 0x1.6a09e667f3bcdp+0) { f = f * 0.5; e += 1; }
    const double s = (f - 1.0) / (f + 1.0);
    const double s2 = s * s;
    double t = 0x1.642c8590b2164p-4;
    t = fma(t, s2, 0x1.8618618618618p-4);
    t = fma(t, s2, 0x1.af286bca1af28p-4);
    t = fma(t, s2, 0x1.e1e1e1e1e1e1ep-4);
    t = fma(t, s2, 0x1.1111111111111p-3);
    t = fma(t, s2, 0x1.3b13b13b13b14p-3);
    t = fma(t, s2, 0x1.745d1745d1746p-3);
    t = fma(t, s2, 0x1.c71c71c71c71cp-3);
    t = fma(t, s2, 0x1.2492492492492p-2);
    t = fma(t, s2, 0x1.999999999999ap-2);
    t = fma(t, s2, 0x1.5555555555555p-1);
    t = fma(t, s2, 0x1.0p+1);
    const double lf = s * t;
    return fma((double)e, 0x1.62e42fefa39efp-1, lf);
}

/* ------------------------------------------------------------------------ */
/* Philox4x32-10 (Salmon, Moraes, Dror & Shaw, SC'11, "Parallel random       */
/* numbers: as easy as 1, 2, 3")                                             */
/* ------------------------------------------------------------------------ */

void orc_philox4x32_10(const uint32_t ctr_in[4], const uint32_t key_in[2], uint32_t out[4])
{
    uint32_t c0 = ctr_in[0], c1 = ctr_in[1], c2 = ctr_in[2], c3 = ctr_in[3];
    uint32_t k0 = key_in[0], k1 = key_in[1];
    for (int i = 0; i < 10; ++i) {
        const uint64_t p0 = (uint64_t)0xD2511F53u * c0;
        const uint64_t p1 = (uint64_t)0xCD9E8D57u * c2;
        const uint32_t hi0 = (uint32_t)(p0 >> 32), lo0 = (uint32_t)p0;
        const uint32_t hi1 = (uint32_t)(p1 >> 32), lo1 = (uint32_t)p1;
        const uint32_t n0 = hi1 ^ c1 ^ k0, n1 = lo1, n2 = hi0 ^ c3 ^ k1, n3 = lo0;
        c0 = n0; c1 = n1; c2 = n2; c3 = n3;
        k0 += 0x9E3779B9u;
        k1 += 0xBB67AE85u;
    }
    out[0] = c0; out[1] = c1; out[2] = c2; out[3] = c3;
}

/* Random word for (row, token) under (seed, offset): counter
 * {token / 4, row, offset_lo, offset_hi}, key {seed_lo, seed_hi}, word token % 4. */
static uint32_t orc_word(uint64_t seed, uint64_t offset, uint32_t row, uint32_t token)
{
    const uint32_t ctr[4] = {token >> 2, row, (uint32_t)offset, (uint32_t)(offset >> 32)};
    const uint32_t key[2] = {(uint32_t)seed, (uint32_t)(seed >> 32)};
    uint32_t o[4];
    orc_philox4x32_10(ctr, key, o);
    return o[token & 3];
}

/* Gumbel value from a 32-bit word: u = (w + 1/2) 2^-32, g = -log(-log u),
 * in fp64 with orc_log64, rounded to fp32. */
float orc_gumbel_from_word(uint32_t w)
{
    const double u = ((double)w + 0.5) * 0x1p-32;
    return (float)(-orc_log64(-orc_log64(u)));
}

/* 53-bit uniform integer for (row, stream) under (seed, offset): counter
 * {0xFFFFFFFF, row, offset_lo, offset_hi} with key {seed_lo, seed_hi ^ stream};
 * the top 53 bits of (w0 << 32 | w1). */
uint64_t orc_u53(uint64_t seed, uint64_t offset, uint32_t row, uint32_t stream)
{
    const uint32_t ctr[4] = {0xFFFFFFFFu, row, (uint32_t)offset, (uint32_t)(offset >> 32)};
    const uint32_t key[2] = {(uint32_t)seed, (uint32_t)(seed >> 32) ^ stream};
    uint32_t o[4];
    orc_philox4x32_10(ctr, key, o);
    return (((uint64_t)o[0] << 32) | o[1]) >> 11;
}

/* A uniform in [0,1) given as fp64 becomes the integer floor(u 2^53). */
static uint64_t orc_u53_from_double(double u)
{
    if (!(u > 0.0)) return 0;
    if (u >= 1.0) return (1ULL << 53) - 1;
    return (uint64_t)(u * 0x1p53);
}

/* floor(u53 * w / 2^53) for w < 2^64, via 128-bit arithmetic. */
static uint64_t orc_scale_u53(uint64_t u53, uint64_t w)
{
    const unsigned __int128 p = (unsigned __int128)(u53 << 11) * w;
    return (uint64_t)(p >> 64);
}

/* ------------------------------------------------------------------------ */
/* Ranking key: (logit desc, token asc).  -0.0 is folded into +0.0 first.    */
/* ------------------------------------------------------------------------ */

static inline uint32_t orc_ordkey(float x)
{
    float y = x + 0.0f;
    uint32_t u;
    memcpy(&u, &y, 4);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

static inline uint64_t orc_rankkey(float x, uint32_t idx)
{
    return ((uint64_t)orc_ordkey(x) << 32) | (uint64_t)(0xFFFFFFFFu - idx);
}

static inline float orc_key_value(uint64_t key)
{
    const uint32_t o = (uint32_t)(key >> 32);
    const uint32_t u = (o & 0x80000000u) ? (o & 0x7FFFFFFFu) : ~o;
    float x;
    memcpy(&x, &u, 4);
    return x;
}

static inline uint32_t orc_key_index(uint64_t key)
{
    return 0xFFFFFFFFu - (uint32_t)key;
}

/* ------------------------------------------------------------------------ */
/* Logits processors                                                        */
/* ------------------------------------------------------------------------ */

/* Start of a processor's window within a history of length H, with Python's
 * `tokens[-context_size:]` meaning (mlx-lm processors slice the running
 * sequence this way; the reference hands them the sequence at
 * verify_decode.py:828-831 and :891-896). */
static int orc_window_start(int H, int ctx)
{
    if (ctx > 0) return H > ctx ? H - ctx : 0;
    if (ctx == 0) return 0;
    return (-ctx) < H ? -ctx : H;
}

typedef struct orc_proc {
    float rep_penalty;  int32_t rep_ctx;  int32_t rep_on;
    float pres_penalty; int32_t pres_ctx; int32_t pres_on;
    float freq_penalty; int32_t freq_ctx; int32_t freq_on;
} orc_proc;

/* Apply, in mlx-lm's make_logits_processors order, logit_bias, then the
 * repetition, presence and frequency penalties, then the allowed-token
 * bitmask, to one row in place.
 *   repetition: each distinct id in its window once, x<0 ? x*pen : x/pen
 *               (mlx-lm make_repetition_penalty; pinned only relative to
 *               mlx-lm by reference tests/test_verify_decode.py:196-203);
 *   presence:   each distinct id in its window once, x - pen;
 *   frequency:  each distinct id in its window once, x - pen*count where
 *               count is its occurrences in that window (product rounded
 *               once);
 *   bitmask:    where(bit, x, -inf), bit v = word v/32 bit v%32 -- the
 *               general form of think_budget.py:107-109 and rescue.py:240-245.
 * Ids outside [0, V) are ignored.  `stamp` is caller scratch of V ints. */
void orc_apply_processors(float *x, int V, const int32_t *hist, int H, const orc_proc *pp,
                          const int32_t *bias_tok, const float *bias_val, int n_bias,
                          const uint32_t *mask, int *stamp)
{
    for (int b = 0; b < n_bias; ++b) {
        const int t = bias_tok[b];
        if (t >= 0 && t < V) x[t] = x[t] + bias_val[b];
    }
    if (H > 0 && pp) {
        if (pp->rep_on) {
            const int s = orc_window_start(H, pp->rep_ctx);
            for (int i = s; i < H; ++i) { const int t = hist[i]; if (t >= 0 && t < V) stamp[t] = 0; }
            for (int i = s; i < H; ++i) {
                const int t = hist[i];
                if (t < 0 || t >= V || stamp[t]) continue;
                stamp[t] = 1;
                const float v = x[t];
                x[t] = v < 0.0f ? v * pp->rep_penalty : v / pp->rep_penalty;
            }
        }
        if (pp->pres_on) {
            const int s = orc_window_start(H, pp->pres_ctx);
            for (int i = s; i < H; ++i) { const int t = hist[i]; if (t >= 0 && t < V) stamp[t] = 0; }
            for (int i = s; i < H; ++i) {
                const int t = hist[i];
                if (t < 0 || t >= V || stamp[t]) continue;
                stamp[t] = 1;
                x[t] = x[t] - pp->pres_penalty;
            }
        }
        if (pp->freq_on) {
            const int s = orc_window_start(H, pp->freq_ctx);
            for (int i = s; i < H; ++i) { const int t = hist[i]; if (t >= 0 && t < V) stamp[t] = 0; }
            for (int i = s; i < H; ++i) { const int t = hist[i]; if (t >= 0 && t < V) stamp[t] += 1; }
            for (int i = s; i < H; ++i) {
                const int t = hist[i];
                if (t < 0 || t >= V || stamp[t] <= 0) continue;
                const float cnt = (float)stamp[t];
                stamp[t] = 0;
                x[t] = x[t] - pp->freq_penalty * cnt;
            }
        }
    }
    if (mask) {
        for (int v = 0; v < V; ++v)
            if (!((mask[v >> 5] >> (v & 31)) & 1u)) x[v] = -INFINITY;
    }
}

/* ------------------------------------------------------------------------ */
/* Row log-sum-exp                                                          */
/* ------------------------------------------------------------------------ */

/* Per-tile statistics of one segment: m_t = max, s_t = sum floor(e^(x-m_t) 2^52). */
void orc_tile_stats(const float *x, int V, float *m_out, uint64_t *s_out)
{
    const int nt = (V + ORC_TILE - 1) / ORC_TILE;
    for (int t = 0; t < nt; ++t) {
        const int a = t * ORC_TILE, b = a + ORC_TILE < V ? a + ORC_TILE : V;
        float m = -INFINITY;
        for (int i = a; i < b; ++i) if (x[i] > m) m = x[i];
        uint64_t s = 0;
        if (m > -INFINITY)
            for (int i = a; i < b; ++i) s += orc_q52(x[i] - m);
        m_out[t] = m;
        s_out[t] = s;
    }
}

static double orc_pairwise(double *a, int n)
{
    int p = 1;
    while (p < n) p <<= 1;
    for (int i = n; i < p; ++i) a[i] = 0.0;
    for (int w = p; w > 1; w >>= 1)
        for (int i = 0; i < w / 2; ++i) a[i] = a[2 * i] + a[2 * i + 1];
    return a[0];
}

/* Combine tile statistics into c = fl32(m + log(Z 2^-52)), m = max m_t,
 * Z = pairwise-sum_t s_t e^(m_t - m).  -inf when every tile is empty. */
float orc_combine_tiles(const float *m_t, const uint64_t *s_t, int nt)
{
    float m = -INFINITY;
    for (int t = 0; t < nt; ++t) if (m_t[t] > m) m = m_t[t];
    if (!(m > -INFINITY)) return -INFINITY;
    int p = 1;
    while (p < nt) p <<= 1;
    double *a = (double *)malloc(sizeof(double) * (size_t)p);
    for (int t = 0; t < nt; ++t)
        a[t] = s_t[t] ? (double)s_t[t] * orc_exp64((double)m_t[t] - (double)m) : 0.0;
    const double Z = orc_pairwise(a, nt);
    free(a);
    return (float)((double)m + orc_log64(Z * 0x1p-52));
}

float orc_row_lse(const float *x, int V)
{
    const int nt = (V + ORC_TILE - 1) / ORC_TILE;
    float *m = (float *)malloc(sizeof(float) * (size_t)nt);
    uint64_t *s = (uint64_t *)malloc(sizeof(uint64_t) * (size_t)nt);
    orc_tile_stats(x, V, m, s);
    const float c = orc_combine_tiles(m, s, nt);
    free(m);
    free(s);
    return c;
}

/* ------------------------------------------------------------------------ */
/* Sampler                                                                  */
/* ------------------------------------------------------------------------ */

typedef struct orc_sampler {
    int32_t greedy;          /* temperature == 0 */
    float inv_temp;          /* fl32(1/temperature) */
    int32_t top_k;           /* > 0: on */
    int32_t top_p_on;        /* 0 < top_p < 1 */
    float top_p_comp;        /* fl32(1 - top_p) */
    int32_t min_p_on;        /* min_p != 0 */
    float log_min_p;         /* fl32(log(min_p)) */
    int32_t min_keep;        /* min_tokens_to_keep */
} orc_sampler;

typedef struct orc_noise {
    int32_t mode;            /* 0: injected, 1: philox */
    const float *gumbel;     /* injected: Gumbel values of this row, [V] */
    const double *uniform;   /* injected: two uniforms of this row, [2] */
    uint64_t seed, offset;   /* philox */
    uint32_t row;            /* philox row id */
} orc_noise;

static float orc_row_gumbel(const orc_noise *nz, uint32_t token)
{
    if (nz->mode == 0) return nz->gumbel[token];
    return orc_gumbel_from_word(orc_word(nz->seed, nz->offset, nz->row, token));
}

static uint64_t orc_row_u53(const orc_noise *nz, int stream)
{
    if (nz->mode == 0) return orc_u53_from_double(nz->uniform[stream]);
    return orc_u53(nz->seed, nz->offset, nz->row, (uint32_t)stream);
}

static int cmp_desc_u64(const void *a, const void *b)
{
    const uint64_t x = *(const uint64_t *)a, y = *(const uint64_t *)b;
    return x < y ? 1 : (x > y ? -1 : 0);
}

/* Top-n rank keys of the finite entries of x, descending; returns the count. */
static int orc_topn(const float *x, int V, int n, uint64_t *out)
{
    /* min-heap of size n over the rank keys */
    int sz = 0;
    for (int i = 0; i < V; ++i) {
        if (!(x[i] > -INFINITY)) continue;
        const uint64_t k = orc_rankkey(x[i], (uint32_t)i);
        if (sz < n) {
            int j = sz++;
            out[j] = k;
            while (j > 0) {
                const int pj = (j - 1) / 2;
                if (out[pj] <= out[j]) break;
                const uint64_t t = out[pj]; out[pj] = out[j]; out[j] = t;
                j = pj;
            }
        } else if (k > out[0]) {
            out[0] = k;
            int j = 0;
            for (;;) {
                const int l = 2 * j + 1, r = l + 1;
                int s = j;
                if (l < sz && out[l] < out[s]) s = l;
                if (r < sz && out[r] < out[s]) s = r;
                if (s == j) break;
                const uint64_t t = out[s]; out[s] = out[j]; out[j] = t;
                j = s;
            }
        }
    }
    qsort(out, (size_t)sz, sizeof(uint64_t), cmp_desc_u64);
    return sz;
}

/* Whole-vocabulary draw (no filter active): two-level inverse CDF at
 * temperature.  y = fl32(x * inv_temp); per tile (my_t, sy_t) as for the
 * log-sum-exp; tile weights w_t = floor(sy_t e^(my_t - my) 2^-sh) with
 * sh = ceil(log2 n_tiles) + 1; the first uniform picks the tile with
 * target floor(u1 W), the second the token inside the tile with target
 * floor(u2 sy_t), each the first whose inclusive prefix exceeds its target. */
static int32_t orc_full_draw(const float *x, int V, float inv_temp, const orc_noise *nz)
{
    const int nt = (V + ORC_TILE - 1) / ORC_TILE;
    float *y = (float *)malloc(sizeof(float) * (size_t)V);
    if (!y) return 0;
    for (int i = 0; i < V; ++i) y[i] = (x[i] > -INFINITY) ? x[i] * inv_temp : -INFINITY;
    float *m = (float *)malloc(sizeof(float) * (size_t)nt);
    uint64_t *s = (uint64_t *)malloc(sizeof(uint64_t) * (size_t)nt);
    orc_tile_stats(y, V, m, s);
    float mm = -INFINITY;
    for (int t = 0; t < nt; ++t) if (m[t] > mm) mm = m[t];
    int32_t tok = 0;
    if (mm > -INFINITY) {
        int sh = 1;
        while ((1 << (sh - 1)) < nt) ++sh;
        uint64_t *w = (uint64_t *)malloc(sizeof(uint64_t) * (size_t)nt);
        uint64_t W = 0;
        for (int t = 0; t < nt; ++t) {
            const double a = s[t] ? (double)s[t] * orc_exp64((double)m[t] - (double)mm) : 0.0;
            w[t] = (uint64_t)ldexp(a, -sh);
            W += w[t];
        }
        const uint64_t t1 = orc_scale_u53(orc_row_u53(nz, 0), W);
        int tt = nt - 1;
        uint64_t acc = 0;
        for (int t = 0; t < nt; ++t) { acc += w[t]; if (acc > t1) { tt = t; break; } }
        const uint64_t t2 = orc_scale_u53(orc_row_u53(nz, 1), s[tt]);
        const int a = tt * ORC_TILE, b = a + ORC_TILE < V ? a + ORC_TILE : V;
        acc = 0;
        tok = a;
        for (int i = a; i < b; ++i) {
            acc += orc_q52(y[i] - m[tt]);
            if (acc > t2) { tok = i; break; }
        }
        free(w);
    }
    free(y); free(m); free(s);
    return tok;
}

/* One row through the sampler (mlx-lm make_sampler chain: top_k, top_p,
 * min_p, then the categorical draw at temperature; temperature 0 is argmax
 * over the row, reference verify_decode.py:751-752 / lookup_decode.py:359).
 * x is the processed logits row.  lse is the row's log-sum-exp (may be NaN
 * when no filter needs it).  Survivors (ids, renormalised probabilities at
 * temperature) are written in rank order when surv_cap > 0.
 * Returns the number of survivors (0 for greedy / whole-vocabulary draws). */
int orc_sample_row(const float *x, int V, float lse, const orc_sampler *sp, const orc_noise *nz,
                   int32_t *token, int32_t *surv_ids, float *surv_probs, int surv_cap)
{
    if (sp->greedy) {
        int best = 0;
        for (int i = 1; i < V; ++i) if (x[i] > x[best]) best = i;
        *token = best;
        return 0;
    }
    const int filt = sp->top_k > 0 || sp->top_p_on || sp->min_p_on;
    if (!filt) {
        *token = orc_full_draw(x, V, sp->inv_temp, nz);
        return 0;
    }
    int n = V;
    if (sp->top_k > 0 && sp->top_k < n) n = sp->top_k;
    uint64_t *keys = (uint64_t *)malloc(sizeof(uint64_t) * (size_t)(n > 0 ? n : 1));
    int cnt = orc_topn(x, V, n, keys);
    if (cnt == 0) { *token = 0; free(keys); return 0; }
    /* top_p over the survivors of top_k: keep rank r while T - A_r > Q_thr,
     * T = exact sum of their q52 masses when top_k is on, else 2^52. */
    if (sp->top_p_on) {
        uint64_t T = 0;
        uint64_t *q = (uint64_t *)malloc(sizeof(uint64_t) * (size_t)cnt);
        for (int r = 0; r < cnt; ++r) { q[r] = orc_q52(orc_key_value(keys[r]) - lse); T += q[r]; }
        if (sp->top_k <= 0) T = 1ULL << 52;
        const uint64_t qthr = (uint64_t)(sp->top_p_comp * 0x1p52f);
        uint64_t A = 0;
        int keep = 0;
        for (int r = 0; r < cnt; ++r) {
            if (A < T && T - A > qthr) keep = r + 1; else break;
            A += q[r];
        }
        if (keep < 1) keep = 1;
        cnt = keep;
        free(q);
    }
    /* min_p: drop lp < fl32(lp_top + log(min_p)), first min_keep ranks kept. */
    if (sp->min_p_on) {
        const float thr = (orc_key_value(keys[0]) - lse) + sp->log_min_p;
        int keep = cnt;
        for (int r = 0; r < cnt; ++r) {
            if (r >= sp->min_keep && (orc_key_value(keys[r]) - lse) < thr) { keep = r; break; }
        }
        if (keep < 1) keep = 1;
        cnt = keep;
    }
    /* Gumbel-max over the survivors: argmax fl32(fl32(x * inv_temp) + g), ties to the lowest id. */
    int32_t best = -1;
    float bs = -INFINITY;
    for (int r = 0; r < cnt; ++r) {
        const uint32_t id = orc_key_index(keys[r]);
        const float sc = orc_key_value(keys[r]) * sp->inv_temp + orc_row_gumbel(nz, id);
        if (best < 0 || sc > bs || (sc == bs && (int32_t)id < best)) { bs = sc; best = (int32_t)id; }
    }
    *token = best;
    if (surv_cap > 0) {
        double ymax = -INFINITY;
        for (int r = 0; r < cnt; ++r) {
            const double yv = (double)(orc_key_value(keys[r]) * sp->inv_temp);
            if (yv > ymax) ymax = yv;
        }
        double Z = 0.0;
        for (int r = 0; r < cnt; ++r) Z += orc_exp64((double)(orc_key_value(keys[r]) * sp->inv_temp) - ymax);
        for (int r = 0; r < cnt && r < surv_cap; ++r) {
            surv_ids[r] = (int32_t)orc_key_index(keys[r]);
            surv_probs[r] = (float)(orc_exp64((double)(orc_key_value(keys[r]) * sp->inv_temp) - ymax) / Z);
        }
    }
    free(keys);
    return cnt;
}

/* Batched driver: processors, log-sum-exp and sampler for B rows.  hist is [B, hist_stride] with per-row lengths; mask is
 * [B, mask_stride] words or NULL; gumbel [B, V] / uniform [B, 2] for injected
 * noise.  lse_out [B] receives each row's log-sum-exp. */
int orc_sample_batch(const float *logits, int B, int V, const int32_t *hist, int hist_stride,
                     const int32_t *hist_len, const orc_proc *pp, const int32_t *bias_tok,
                     const float *bias_val, int n_bias, const uint32_t *mask, int mask_stride,
                     const orc_sampler *sp, int noise_mode, const float *gumbel, const double *uniform,
                     uint64_t seed, uint64_t offset, uint32_t row_base, int32_t *tokens, float *lse_out,
                     int32_t *surv_ids, float *surv_probs, int32_t *n_surv, int surv_cap)
{
    if (B < 0 || V <= 0) return ORC_ERR_ARG;
    int err = 0;
    for (int r = 0; r < B; ++r) {
        float *x = (float *)malloc(sizeof(float) * (size_t)V);
        int *stamp = (int *)calloc((size_t)V, sizeof(int));
        if (!x || !stamp) { err = 1; free(x); free(stamp); continue; }
        memcpy(x, logits + (size_t)r * V, sizeof(float) * (size_t)V);
        orc_apply_processors(x, V, hist ? hist + (size_t)r * hist_stride : NULL,
                             hist ? (hist_len ? hist_len[r] : hist_stride) : 0, pp, bias_tok, bias_val,
                             n_bias, mask ? mask + (size_t)r * mask_stride : NULL, stamp);
        const float lse = orc_row_lse(x, V);
        if (lse_out) lse_out[r] = lse;
        orc_noise nz;
        nz.mode = noise_mode;
        nz.gumbel = gumbel ? gumbel + (size_t)r * V : NULL;
        nz.uniform = uniform ? uniform + (size_t)r * 2 : NULL;
        nz.seed = seed;
        nz.offset = offset;
        nz.row = row_base + (uint32_t)r;
        const int ns = orc_sample_row(x, V, lse, sp, &nz, tokens + r,
                                      surv_ids ? surv_ids + (size_t)r * surv_cap : NULL,
                                      surv_probs ? surv_probs + (size_t)r * surv_cap : NULL,
                                      surv_ids ? surv_cap : 0);
        if (n_surv) n_surv[r] = ns;
        free(x);
        free(stamp);
    }
    return err ? ORC_ERR_ARG : ORC_OK;
}

/* Processors then row-wise log-softmax: out = x - lse(x) (reference
 * verify_decode.py:835, :899; lookup_decode.py:358). */
int orc_logprobs_batch(const float *logits, int B, int V, const int32_t *hist, int hist_stride,
                       const int32_t *hist_len, const orc_proc *pp, const int32_t *bias_tok,
                       const float *bias_val, int n_bias, const uint32_t *mask, int mask_stride,
                       float *out, float *lse_out)
{
    for (int r = 0; r < B; ++r) {
        float *x = out + (size_t)r * V;
        int *stamp = (int *)calloc((size_t)V, sizeof(int));
        memcpy(x, logits + (size_t)r * V, sizeof(float) * (size_t)V);
        orc_apply_processors(x, V, hist ? hist + (size_t)r * hist_stride : NULL,
                             hist ? (hist_len ? hist_len[r] : hist_stride) : 0, pp, bias_tok, bias_val,
                             n_bias, mask ? mask + (size_t)r * mask_stride : NULL, stamp);
        const float lse = orc_row_lse(x, V);
        if (lse_out) lse_out[r] = lse;
        for (int i = 0; i < V; ++i) x[i] = x[i] - lse;
        free(stamp);
    }
    return ORC_OK;
}

/* Processors only (the logits-processor callables' output). */
int orc_process_batch(const float *logits, int B, int V, const int32_t *hist, int hist_stride,
                      const int32_t *hist_len, const orc_proc *pp, const int32_t *bias_tok,
                      const float *bias_val, int n_bias, const uint32_t *mask, int mask_stride,
                      float *out)
{
    for (int r = 0; r < B; ++r) {
        float *x = out + (size_t)r * V;
        int *stamp = (int *)calloc((size_t)V, sizeof(int));
        memcpy(x, logits + (size_t)r * V, sizeof(float) * (size_t)V);
        orc_apply_processors(x, V, hist ? hist + (size_t)r * hist_stride : NULL,
                             hist ? (hist_len ? hist_len[r] : hist_stride) : 0, pp, bias_tok, bias_val,
                             n_bias, mask ? mask + (size_t)r * mask_stride : NULL, stamp);
        free(stamp);
    }
    return ORC_OK;
}

/* Vector form used by the residual-mode restatement: out[i] =
 * orc_expf(fl32(x[i] - c)) (0 for x[i] = -inf), the probabilities
 * expf(y - lse(y)) of a whole row in one call. */
void orc_expf_shift(const float *x, int n, float c, float *out)
{
    for (int i = 0; i < n; ++i) {
        const float d = x[i] - c;
        out[i] = orc_expf(d);
    }
}
