/*
 * sv_oracle.c -- CPU restatement of StarVector's per-token decode-sampling step.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA kernels
 * of comfyui-starvector-gguf_b200 and the CPU baseline timed by bench.py.  No product
 * code path links or calls it.
 *
 * It restates, step by step and sequentially, the reference's sampling chain
 * (ComfyUI-StarVector-GGUF, runtime_shared.py):
 *   _penalize            runtime_shared.py:170-173
 *   _warp                runtime_shared.py:176-187  (temperature, top-k, top-p)
 *   _sample draw line    runtime_shared.py:200-202
 *   _beam_sample step    runtime_shared.py:230-237  (log_softmax, warp, + running
 *                                                    scores, softmax over beams*V,
 *                                                    draw without replacement)
 *   _repeating           runtime_shared.py:156-167
 *
 * The arithmetic is the specification shared with the kernels:
 *   - penalty and temperature are IEEE fp32 multiplications/divisions, exactly as
 *     torch's CPU kernels perform them;
 *   - exp(x) is computed by sv_exp below (Cody-Waite reduction + degree-7 Taylor
 *     polynomial, Horner with fused multiply-add), identical on CPU and GPU;
 *   - every sum that decides something (log-softmax normaliser, top-p cumulative
 *     mass, the draw) is an exact 64-bit fixed-point sum of weights
 *     W = trunc(w * 2^44), so the result does not depend on summation order;
 *   - ties in the ascending top-p sort are ordered by vocabulary index (torch's CPU
 *     sort is unstable, so the reference's order inside a tie is unspecified);
 *   - the draw is an inverse CDF over the kept tokens in ascending vocabulary index
 *     (flattened beam*V index in beam mode) against a supplied uniform u in [0,1):
 *     the first index whose inclusive prefix weight exceeds floor(u * total).
 *
 * Build: gcc -O2 -ffp-contract=off -fno-fast-math -fopenmp -shared -fPIC
 * (oracle/build.py).  -ffp-contract=off matters: only the explicit fmaf/fma calls
 * may fuse, as in the CUDA code.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

enum {
    ORC_OK = 0,
    ORC_ERR_NAN = 1,        /* a NaN logit: the reference's multinomial raises */
    ORC_ERR_POSINF = 2,     /* +inf after penalty/temperature: softmax gives NaN */
    ORC_ERR_ALLNEGINF = 3,  /* no finite logit in the row */
    ORC_ERR_HISTORY = 4,    /* a history id outside [0, V) */
    ORC_ERR_ARGS = 5,
};

/* ------------------------------------------------------------------ helpers */

static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* Order-preserving map float -> uint32 (larger float -> larger key). */
static inline uint32_t ord_key(float f)
{
    uint32_t u = f2u(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

/* exp(x): Cody-Waite argument reduction x = n*ln2 + r, |r| <= ln2/2, then the
 * degree-7 Taylor polynomial of e^r (coefficients 1/k!) in Horner form with fused
 * multiply-add, then scaling by 2^n (two steps below 2^-126 so a subnormal result
 * is rounded once).  Max error about 1.5 ulp against the true exponential. */
float orc_exp(float x)
{
    if (x != x) return x;
    if (x > 88.72283935546875f) return INFINITY;
    if (x < -104.0f) return 0.0f;
    float j = rintf(x * 1.44269502162933349609375f);
    int n = (int)j;
    // ln 2 split in two floats, as SLEEF's single-precision L2Uf / L2Lf (Cody-Waite):
    // the high part has few mantissa bits, so j times it is exact over the j used here.
    float r = fmaf(-j, 0.693145751953125f, x);
    r = fmaf(-j, 1.428606765330187045e-06f, r);
    float p = 1.98412698412698412698e-4f;
    p = fmaf(p, r, 1.38888888888888888889e-3f);
    p = fmaf(p, r, 8.33333333333333333333e-3f);
    p = fmaf(p, r, 4.16666666666666666667e-2f);
    p = fmaf(p, r, 1.66666666666666666667e-1f);
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    if (n > 127) { p = p * 2.0f; n -= 1; }
    if (n >= -126) return p * u2f((uint32_t)(n + 127) << 23);
    return (p * u2f((uint32_t)(n + 127 + 64) << 23)) * u2f((uint32_t)(127 - 64) << 23);
}

/* Fixed-point weight of w in [0,1]: trunc(w * 2^44). */
static inline uint64_t fixw(float w) { return (uint64_t)(w * 17592186044416.0f); }

/* floor(a * f) for f in [0,1), exact (128-bit product of a and f's significand). */
uint64_t orc_mulfloor(uint64_t a, float f)
{
    if (!(f > 0.0f)) return 0;
    if (f >= 1.0f) f = u2f(0x3f7fffffu);
    uint32_t b = f2u(f);
    int ex = (int)((b >> 23) & 0xffu);
    uint64_t mant = b & 0x7fffffu;
    int sh;
    if (ex == 0) sh = 149;
    else { mant |= 0x800000u; sh = 150 - ex; }
    unsigned __int128 prod = (unsigned __int128)a * mant;
    if (sh >= 128) return 0;
    return (uint64_t)(prod >> sh);
}

/* ln(sw * 2^-44) rounded to float, sw >= 1.  Double-precision evaluation:
 * sw = m * 2^e with m in [sqrt(1/2), sqrt(2)), ln m = 2 atanh(z) with
 * z = (m-1)/(m+1), series 2z * sum_{j=0..11} z^(2j)/(2j+1) in Horner form. */
float orc_log_fixed(uint64_t sw)
{
    double d = (double)sw;
    int e;
    double m = frexp(d, &e);
    if (m < 0.70710678118654752440) { m = m * 2.0; e -= 1; }
    double z = (m - 1.0) / (m + 1.0);
    double z2 = z * z;
    double p = 1.0 / 23.0;
    p = fma(p, z2, 1.0 / 21.0);
    p = fma(p, z2, 1.0 / 19.0);
    p = fma(p, z2, 1.0 / 17.0);
    p = fma(p, z2, 1.0 / 15.0);
    p = fma(p, z2, 1.0 / 13.0);
    p = fma(p, z2, 1.0 / 11.0);
    p = fma(p, z2, 1.0 / 9.0);
    p = fma(p, z2, 1.0 / 7.0);
    p = fma(p, z2, 1.0 / 5.0);
    p = fma(p, z2, 1.0 / 3.0);
    p = fma(p, z2, 1.0);
    double lm = (z + z) * p;
    double r = fma((double)(e - 44), 0.69314718055994530942, lm);
    return (float)r;
}

/* k-th largest (1-based) of a[0..n) by quickselect; a is permuted. */
static float kth_largest(float *a, int64_t n, int64_t k)
{
    int64_t lo = 0, hi = n - 1, want = k - 1;
    while (lo < hi) {
        float pv = a[lo + (hi - lo) / 2];
        int64_t i = lo, j = hi;
        while (i <= j) {
            while (a[i] > pv) i++;
            while (a[j] < pv) j--;
            if (i <= j) { float t = a[i]; a[i] = a[j]; a[j] = t; i++; j--; }
        }
        if (want <= j) hi = j;
        else if (want >= i) lo = i;
        else return a[want];
    }
    return a[want];
}

/* Stable LSD radix sort of indices 0..n-1 by 32-bit keys, ascending.  Because
 * it starts from index order and is stable, equal keys stay in index order. */
static void radix_sort_idx(const uint32_t *key, int64_t n, uint32_t *idx, uint32_t *tmp)
{
    for (int64_t i = 0; i < n; i++) idx[i] = (uint32_t)i;
    int64_t cnt[256];
    for (int pass = 0; pass < 4; pass++) {
        int sh = pass * 8;
        memset(cnt, 0, sizeof cnt);
        for (int64_t i = 0; i < n; i++) cnt[(key[idx[i]] >> sh) & 0xff]++;
        int64_t s = 0;
        for (int b = 0; b < 256; b++) { int64_t c = cnt[b]; cnt[b] = s; s += c; }
        for (int64_t i = 0; i < n; i++) tmp[cnt[(key[idx[i]] >> sh) & 0xff]++] = idx[i];
        memcpy(idx, tmp, (size_t)n * sizeof(uint32_t));
    }
}

/* Working memory for one row. */
typedef struct {
    int64_t cap;
    float *s, *sel;
    uint32_t *key, *idx, *tmp;
} work_t;

static int work_reserve(work_t *w, int64_t V)
{
    if (w->cap >= V) return 0;
    free(w->s); free(w->sel); free(w->key); free(w->idx); free(w->tmp);
    w->s = malloc((size_t)V * 4); w->sel = malloc((size_t)V * 4);
    w->key = malloc((size_t)V * 4); w->idx = malloc((size_t)V * 4); w->tmp = malloc((size_t)V * 4);
    w->cap = V;
    return (w->s && w->sel && w->key && w->idx && w->tmp) ? 0 : -1;
}

static void work_free(work_t *w)
{
    free(w->s); free(w->sel); free(w->key); free(w->idx); free(w->tmp);
    memset(w, 0, sizeof *w);
}

/*
 * _warp(_penalize(scores, seen), T, top_p, keep) in place on s[0..V):
 * runtime_shared.py:170-187.  On return s holds the warped scores (-inf where
 * masked).  *pmax receives the row maximum M (the maximum of the warped scores).
 *   pen: seen ? (s < 0 ? s*rp : s/rp) : s            (:172-173)
 *   temperature: s / T, then -0 -> +0                 (:178-179; x/1 == x)
 *   top-k: thr = kk-th largest, s < thr -> -inf       (:180-181)
 *   top-p: ascending sort, softmax, cumsum <= 1-top_p removed,
 *          last `keep` never removed, scatter back     (:182-186)
 */
static int warp_row(work_t *w, float *s, int64_t V, const uint8_t *seen, float T, float rp,
                    float pthr, int kk, int keep, float *pmax)
{
    /* A NaN anywhere in the row takes precedence over +inf (either makes the
     * reference's multinomial raise; the status only names the cause). */
    int any_nan = 0, any_inf = 0;
    for (int64_t i = 0; i < V; i++) {
        float v = s[i];
        if (seen && seen[i]) v = (v < 0.0f) ? v * rp : v / rp;
        /* Temperature, then -0 -> +0: torch compares -0 == +0, and the canonical
         * zero keeps the ordered-key sort consistent with float comparisons. */
        v = v / T + 0.0f;
        any_nan |= v != v;
        any_inf |= v == INFINITY;
        s[i] = v;
    }
    if (any_nan) return ORC_ERR_NAN;
    if (any_inf) return ORC_ERR_POSINF;
    memcpy(w->sel, s, (size_t)V * 4);
    float thr = kth_largest(w->sel, V, kk);
    float M = -INFINITY;
    for (int64_t i = 0; i < V; i++) {
        if (s[i] < thr) s[i] = -INFINITY;
        if (s[i] > M) M = s[i];
    }
    if (M == -INFINITY) return ORC_ERR_ALLNEGINF;
    *pmax = M;
    if (pthr > 0.0f) {
        for (int64_t i = 0; i < V; i++) w->key[i] = ord_key(s[i]);
        radix_sort_idx(w->key, V, w->idx, w->tmp);
        uint64_t total = 0;
        for (int64_t i = 0; i < V; i++) total += fixw(orc_exp(s[i] - M));
        uint64_t thrW = orc_mulfloor(total, pthr);
        uint64_t P = 0;
        int64_t r = 0;
        for (int64_t j = 0; j < V; j++) {
            P += fixw(orc_exp(s[w->idx[j]] - M));
            if (P <= thrW) r = j + 1; else break;
        }
        if (r > V - keep) r = V - keep;
        for (int64_t j = 0; j < r; j++) s[w->idx[j]] = -INFINITY;
    }
    return ORC_OK;
}

/* Draw from the kept (finite) entries of s with weights fixw(exp(s-M)):
 * first index (ascending) whose inclusive prefix exceeds floor(u * total). */
static int64_t draw_row(const float *s, int64_t V, float M, float u, uint64_t *ptotal)
{
    uint64_t total = 0;
    for (int64_t i = 0; i < V; i++)
        if (s[i] > -INFINITY) total += fixw(orc_exp(s[i] - M));
    *ptotal = total;
    uint64_t t = orc_mulfloor(total, u);
    uint64_t c = 0;
    int64_t last = -1;
    for (int64_t i = 0; i < V; i++) {
        if (!(s[i] > -INFINITY)) continue;
        c += fixw(orc_exp(s[i] - M));
        last = i;
        if (c > t) return i;
    }
    return last;
}

static float inv_total(uint64_t total) { return (float)total * 5.684341886080801487e-14f; /* 2^-44 */ }

/*
 * One row of the sample-mode step: runtime_shared.py:200-202 with the draw line
 * replaced by the supplied-uniform rule.
 *   x: fp32 logits [V]; seen: bool bytes [V] or NULL.
 *   Outputs: token; count = number of kept (finite) tokens; the first `cap` kept
 *   (index ascending) into oidx/oprob; optional dense warped scores and probs.
 */
static int sample_row(work_t *w, const float *x, int64_t V, const uint8_t *seen, float T, float rp,
                      float pthr, int kk, int keep, float u, int64_t *token, int32_t *count,
                      int32_t *oidx, float *oprob, int cap, float *dscores, float *dprobs)
{
    if (work_reserve(w, V)) return ORC_ERR_ARGS;
    if (V < kk || kk < 1 || keep < 1) return ORC_ERR_ARGS;
    float *s = w->s;
    memcpy(s, x, (size_t)V * 4);
    float M = 0.0f;
    int st = warp_row(w, s, V, seen, T, rp, pthr, kk, keep, &M);
    if (st != ORC_OK) {
        *token = -1; *count = 0;
        for (int64_t i = 0; i < V; i++) {
            if (dscores) dscores[i] = -INFINITY;
            if (dprobs) dprobs[i] = 0.0f;
        }
        return st;
    }
    uint64_t total;
    *token = draw_row(s, V, M, u, &total);
    float S = inv_total(total);
    int32_t n = 0;
    for (int64_t i = 0; i < V; i++) {
        float q = 0.0f;
        if (s[i] > -INFINITY) {
            q = orc_exp(s[i] - M) / S;
            if (n < cap) { oidx[n] = (int32_t)i; oprob[n] = q; }
            n++;
        }
        if (dscores) dscores[i] = s[i];
        if (dprobs) dprobs[i] = q;
    }
    *count = n;
    return ORC_OK;
}

/* ------------------------------------------------------------- public entry */

/* Sample-mode step over R rows.
 *   logits fp32 [R, row_stride]; history: either `seen` bool bytes [R, V] (if
 *   seen != NULL) or int32 ids [R, hist_stride] with hist_len[R] (if ids != NULL).
 *   temperature, top_p, rep_penalty are doubles cast to float as torch casts a
 *   Python scalar; top-p is active iff top_p < 1 with threshold float(1 - top_p).
 *   Per-row status in status[R]; returns the number of rows with nonzero status.
 */
int orc_sample(const float *logits, int64_t R, int64_t V, int64_t row_stride,
               const uint8_t *seen, const int32_t *ids, const int32_t *hist_len, int64_t hist_stride,
               double temperature, double top_p, int top_k, int keep, double rep_penalty,
               const float *uniforms,
               int64_t *token, int32_t *count, int32_t *oidx, float *oprob, int cap,
               float *dscores, float *dprobs, int32_t *status, int nthreads)
{
    float T = (float)temperature, rp = (float)rep_penalty;
    float pthr = top_p < 1.0 ? (float)(1.0 - top_p) : 0.0f;
    int kk = top_k > keep ? top_k : keep;
    int bad = 0;
#ifdef _OPENMP
    if (nthreads < 1) nthreads = omp_get_max_threads();
#pragma omp parallel num_threads(nthreads) reduction(+ : bad)
#endif
    {
        work_t w = {0};
        uint8_t *mask = NULL;
        if (ids) mask = calloc((size_t)V, 1);
#ifdef _OPENMP
#pragma omp for schedule(dynamic, 1)
#endif
        for (int64_t r = 0; r < R; r++) {
            const uint8_t *sn = seen ? seen + r * V : NULL;
            int st = ORC_OK;
            if (ids) {
                memset(mask, 0, (size_t)V);
                int64_t L = hist_len ? hist_len[r] : hist_stride;
                for (int64_t j = 0; j < L; j++) {
                    int32_t id = ids[r * hist_stride + j];
                    if (id < 0 || id >= V) { st = ORC_ERR_HISTORY; break; }
                    mask[id] = 1;
                }
                sn = mask;
            }
            if (st == ORC_OK)
                st = sample_row(&w, logits + r * row_stride, V, sn, T, rp, pthr, kk, keep, uniforms[r],
                                token + r, count + r, oidx ? oidx + r * cap : NULL, oprob ? oprob + r * cap : NULL,
                                oidx ? cap : 0, dscores ? dscores + r * V : NULL, dprobs ? dprobs + r * V : NULL);
            else { token[r] = -1; count[r] = 0; }
            status[r] = st;
            bad += st != ORC_OK;
        }
        work_free(&w);
        free(mask);
    }
    return bad;
}

/*
 * One beam-sampling step (runtime_shared.py:230-237) for B beams:
 *   log_probs = _warp(_penalize(log_softmax(x), seen), T, top_p, keep)
 *   scores    = log_probs + running[:, None], flattened to [B*V]
 *   probs     = softmax(scores); picks drawn without replacement,
 *               n = min(npick_max, count_nonzero(probs))
 * log_softmax: M = max x, S = sum fixw(exp(x - M)) (exact), L = ln S (orc_log_fixed),
 *   lp = (x - M) - L.
 * Global softmax: M* = max scores, w = exp(scores - M*), Sw* = sum fixw(w),
 *   p = w / (Sw* 2^-44).
 * Draw j: R = entries with p > 0 not yet picked, flattened index order; if the
 *   remaining fixed-point total TW > 0, pick the first with inclusive prefix >
 *   floor(u_j * TW); otherwise the largest p (lowest index on ties).
 * Outputs picks (flattened b*V + i), picked scores, n, plus optional dense
 * warped log-probs [B,V] and probs [B*V], and per-beam max / log-normaliser.
 */
int orc_beam(const float *logits, int64_t B, int64_t V, int64_t row_stride, const uint8_t *seen,
             const float *running, double temperature, double top_p, int top_k, int keep,
             double rep_penalty, int npick_max, const float *uniforms,
             int64_t *picks, float *pscores, int32_t *npicks,
             float *dlogp, float *dprobs, float *bmax, float *blog, int32_t *nnz_out)
{
    float T = (float)temperature, rp = (float)rep_penalty;
    float pthr = top_p < 1.0 ? (float)(1.0 - top_p) : 0.0f;
    int kk = top_k > keep ? top_k : keep;
    int64_t N = B * V;
    if (V < kk || kk < 1 || keep < 1 || B < 1) return ORC_ERR_ARGS;
    work_t w = {0};
    float *sc = malloc((size_t)N * 4);
    uint64_t *W = malloc((size_t)N * 8);
    uint8_t *rem = malloc((size_t)N);
    int st = ORC_OK;
    if (!sc || !W || !rem || work_reserve(&w, V)) { st = ORC_ERR_ARGS; goto done; }
    for (int64_t b = 0; b < B && st == ORC_OK; b++) {
        const float *x = logits + b * row_stride;
        float M = -INFINITY;
        int any_nan = 0, any_inf = 0;
        for (int64_t i = 0; i < V; i++) {
            any_nan |= x[i] != x[i];
            any_inf |= x[i] == INFINITY;
            if (x[i] > M) M = x[i];
        }
        if (any_nan || any_inf) { st = any_nan ? ORC_ERR_NAN : ORC_ERR_POSINF; break; }
        if (M == -INFINITY) { st = ORC_ERR_ALLNEGINF; break; }
        uint64_t S = 0;
        for (int64_t i = 0; i < V; i++) S += fixw(orc_exp(x[i] - M));
        float L = orc_log_fixed(S);
        if (bmax) bmax[b] = M;
        if (blog) blog[b] = L;
        float *s = sc + b * V;
        for (int64_t i = 0; i < V; i++) s[i] = (x[i] - M) - L;
        float Mw;
        st = warp_row(&w, s, V, seen ? seen + b * V : NULL, T, rp, pthr, kk, keep, &Mw);
        if (dlogp) memcpy(dlogp + b * V, s, (size_t)V * 4);
        float rs = running[b];
        for (int64_t i = 0; i < V; i++) s[i] = s[i] + rs;
    }
    if (st != ORC_OK) goto done;
    float Ms = -INFINITY;
    for (int64_t f = 0; f < N; f++) {
        if (sc[f] != sc[f]) { st = ORC_ERR_NAN; goto done; }
        if (sc[f] > Ms) Ms = sc[f];
    }
    if (Ms == -INFINITY || Ms == INFINITY) { st = Ms == INFINITY ? ORC_ERR_POSINF : ORC_ERR_ALLNEGINF; goto done; }
    uint64_t tot = 0;
    for (int64_t f = 0; f < N; f++) { W[f] = fixw(orc_exp(sc[f] - Ms)); tot += W[f]; }
    float Sf = inv_total(tot);
    int32_t nnz = 0;
    for (int64_t f = 0; f < N; f++) {
        float p = orc_exp(sc[f] - Ms) / Sf;
        if (dprobs) dprobs[f] = p;
        rem[f] = p > 0.0f;
        nnz += rem[f];
    }
    if (nnz_out) *nnz_out = nnz;
    int n = npick_max < nnz ? npick_max : nnz;
    for (int j = 0; j < n; j++) {
        uint64_t TW = 0;
        for (int64_t f = 0; f < N; f++) if (rem[f]) TW += W[f];
        int64_t pick = -1;
        if (TW > 0) {
            uint64_t t = orc_mulfloor(TW, uniforms[j]), c = 0;
            for (int64_t f = 0; f < N; f++) {
                if (!rem[f]) continue;
                c += W[f];
                if (c > t) { pick = f; break; }
            }
        } else {
            float best = -1.0f;
            for (int64_t f = 0; f < N; f++) {
                if (!rem[f]) continue;
                float p = orc_exp(sc[f] - Ms) / Sf;
                if (p > best) { best = p; pick = f; }
            }
        }
        rem[pick] = 0;
        picks[j] = pick;
        pscores[j] = sc[pick];
    }
    *npicks = n;
done:
    if (st != ORC_OK) *npicks = 0;
    free(sc); free(W); free(rem);
    work_free(&w);
    return st;
}

/* _repeating (runtime_shared.py:156-167): True iff len >= window*repeats and the
 * last `window` tokens occur at least `repeats` times (overlapping starts allowed,
 * the tail itself counted).  Batched over R rows of int32 tokens. */
int orc_repeating(const int32_t *tokens, int64_t R, int64_t stride, const int32_t *lengths,
                  int window, int repeats, uint8_t *verdict, int nthreads)
{
#ifdef _OPENMP
    if (nthreads < 1) nthreads = omp_get_max_threads();
#pragma omp parallel for num_threads(nthreads) schedule(dynamic, 1)
#endif
    for (int64_t r = 0; r < R; r++) {
        const int32_t *t = tokens + r * stride;
        int64_t L = lengths[r];
        uint8_t v = 0;
        if (L >= (int64_t)window * repeats) {
            const int32_t *tail = t + L - window;
            int count = 0;
            for (int64_t s = 0; s + window <= L; s++) {
                if (t[s] == tail[0] && memcmp(t + s, tail, (size_t)window * 4) == 0) {
                    if (++count == repeats) { v = 1; break; }
                }
            }
        }
        verdict[r] = v;
    }
    return 0;
}

/* Element-wise helpers exposed for the unit tests of the shared arithmetic. */
void orc_exp_vec(const float *x, float *y, int64_t n)
{
    for (int64_t i = 0; i < n; i++) y[i] = orc_exp(x[i]);
}

void orc_log_fixed_vec(const uint64_t *s, float *y, int64_t n)
{
    for (int64_t i = 0; i < n; i++) y[i] = orc_log_fixed(s[i]);
}

void orc_mulfloor_vec(const uint64_t *a, const float *f, uint64_t *y, int64_t n)
{
    for (int64_t i = 0; i < n; i++) y[i] = orc_mulfloor(a[i], f[i]);
}
