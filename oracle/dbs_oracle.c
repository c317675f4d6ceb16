/*
 * CPU oracle for the differentiable beam search hot path.
 *
 * TEST INFRASTRUCTURE ONLY: the parity tests and bench.py's CPU baseline arm
 * use it as the checker. The product (libdbs.so and its kernels) never links,
 * loads or calls it.
 *
 * Restates the scalar semantics of the reference decoder
 * (maged15/differentiable-beam-search-cuda, src/differentiable_beam.cpp).
 * Built with -ffp-contract=off so every float add / multiply / divide is a
 * separately rounded IEEE operation, as in the reference's non-SIMD code.
 */
#include "dbs_oracle.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

static _Thread_local char g_err[256];

static int fail(const char* msg) {
    snprintf(g_err, sizeof(g_err), "%s", msg);
    return 1;
}

const char* oracle_last_error(void) { return g_err; }

/* from_c_options, src/differentiable_beam.cpp:3145-3177: non-positive fields
 * take defaults, eos is verbatim, validate_inputs==0 disables validation. */
void oracle_options_from_c(int beam_size, int eos_token, float selected_temperature,
                           float soft_topk_temperature, int relaxed_pool_multiplier,
                           int vocab_block, float length_penalty_alpha,
                           float soft_topk_tolerance, int soft_topk_max_iters,
                           int min_length, int validate_inputs,
                           int64_t max_dense_gradient_elements, oracle_options* o) {
    o->beam_size = beam_size > 0 ? beam_size : 8;
    o->eos_token = eos_token;
    o->selected_temperature = selected_temperature > 0.0f ? selected_temperature : 1.0f;
    o->soft_topk_temperature = soft_topk_temperature > 0.0f ? soft_topk_temperature : 0.25f;
    o->relaxed_pool_multiplier = relaxed_pool_multiplier > 0 ? relaxed_pool_multiplier : 8;
    o->vocab_block = vocab_block > 0 ? vocab_block : 4096;
    o->length_penalty_alpha = length_penalty_alpha >= 0.0f ? length_penalty_alpha : 0.0f;
    o->soft_topk_tolerance = soft_topk_tolerance > 0.0f ? soft_topk_tolerance : 1.0e-4f;
    o->soft_topk_max_iters = soft_topk_max_iters > 0 ? soft_topk_max_iters : 48;
    o->min_length = min_length >= 0 ? min_length : 0;
    o->validate_inputs = validate_inputs == 0 ? 0 : 1;
    o->max_dense_gradient_elements =
        max_dense_gradient_elements > 0 ? max_dense_gradient_elements : 100000000LL;
    /* DifferentiableBeamSearchAVX512 ctor clamps, :1424-1425 */
    if (o->vocab_block < 16) o->vocab_block = 16;
    if (o->relaxed_pool_multiplier < 1) o->relaxed_pool_multiplier = 1;
}

int oracle_pool_size(const oracle_options* opt) {
    long long p = (long long)opt->beam_size * (long long)opt->relaxed_pool_multiplier;
    return p > opt->beam_size ? (int)p : opt->beam_size; /* :1456-1460 */
}

/* gnmt_length_penalty, :277-282 */
static float gnmt(int length, float alpha) {
    if (alpha == 0.0f) return 1.0f;
    int l = length < 1 ? 1 : length;
    return powf((5.0f + (float)l) / 6.0f, alpha);
}

/* safe_exp_scalar / sigmoid_scalar, :262-275 (std::min/std::max argument
 * order kept, so NaN clamps to the lower bound). */
static float safe_exp(float x) {
    const float hi = 88.3762626647949f;
    x = (-hi < x) ? x : -hi;
    x = (x < hi) ? x : hi;
    return expf(x);
}

static float sigmoid1(float x) {
    if (x >= 0.0f) {
        float e = safe_exp(-x);
        return 1.0f / (1.0f + e);
    }
    float e = safe_exp(x);
    return e / (1.0f + e);
}

typedef struct cand {
    float score;
    float raw;
    int32_t parent;
    int32_t token;
    int32_t length;
    uint8_t flp;
} cand;

/* candidate_better, :291-298 */
static int better(const cand* a, const cand* b) {
    if (a->score != b->score) return a->score > b->score;
    if (a->raw != b->raw) return a->raw > b->raw;
    if (a->parent != b->parent) return a->parent < b->parent;
    if (a->token != b->token) return a->token < b->token;
    if (a->length != b->length) return a->length < b->length;
    return a->flp > b->flp;
}

/* Descending top-n buffer insert (insert_topk, :359-383): the candidate goes
 * after every entry that beats it; the last entry falls off. */
static void push_top(cand* top, int n, const cand* c) {
    if (!better(c, &top[n - 1])) return;
    int lo = 0, hi = n - 1;
    while (lo < hi) {
        int mid = lo + ((hi - lo) >> 1);
        if (better(c, &top[mid])) hi = mid; else lo = mid + 1;
    }
    memmove(&top[lo + 1], &top[lo], (size_t)(n - 1 - lo) * sizeof(cand));
    top[lo] = *c;
}

/* validate_logprob_tensor, :385-402: up to 1000 evenly spaced samples. */
static int validate(const float* x, int steps, int k, int v) {
    size_t count = (size_t)steps * (size_t)k * (size_t)v;
    size_t stride = count > 1000 ? count / 1000 : 1;
    for (size_t i = 0; i < count; i += stride) {
        float value = x[i];
        if (isnan(value) || value == INFINITY) return fail("log_probs contains NaN or +Inf");
    }
    return 0;
}

/* would_repeat_ngram, :305-325 */
static int repeats_ngram(const int32_t* pre, int plen, int token, int n) {
    if (n <= 0) return 0;
    if (n == 1) {
        for (int i = 0; i < plen; ++i) if (pre[i] == token) return 1;
        return 0;
    }
    if (plen + 1 < n) return 0;
    int suffix = plen - (n - 1);
    for (int i = 0; i + n <= plen; ++i) {
        int same = 1;
        for (int j = 0; j < n - 1; ++j) {
            if (pre[i + j] != pre[suffix + j]) { same = 0; break; }
        }
        if (same && pre[i + n - 1] != token) same = 0;
        if (same) return 1;
    }
    return 0;
}

static int prefix_has(const int32_t* pre, int plen, int token) {
    for (int i = 0; i < plen; ++i) if (pre[i] == token) return 1;
    return 0;
}

/* soft_topk_inclusion, :1333-1386 (scalar sum_sigmoid_shifted :444-459 and
 * soft_topk_write :461-474). */
static void soft_topk(const float* s, float* out, int n, int target_k, float temp,
                      float tol, int iters) {
    const float guard = -1.0e30f;
    int active = 0;
    float mn = INFINITY, mx = -INFINITY;
    for (int i = 0; i < n; ++i) {
        out[i] = 0.0f;
        if (s[i] > guard) {
            ++active;
            mn = (s[i] < mn) ? s[i] : mn;
            mx = (mx < s[i]) ? s[i] : mx;
        }
    }
    if (active == 0 || target_k <= 0) return;
    if (target_k >= active) {
        for (int i = 0; i < n; ++i) if (s[i] > guard) out[i] = 1.0f;
        return;
    }
    float lo = mn - 80.0f * temp;
    float hi = mx + 80.0f * temp;
    for (int it = 0; it < iters; ++it) {
        float mid = 0.5f * (lo + hi);
        float sum = 0.0f;
        for (int i = 0; i < n; ++i) if (s[i] > guard) sum += sigmoid1((s[i] - mid) / temp);
        float err = sum - (float)target_k;
        float amid = fabsf(mid);
        if (fabsf(err) <= tol || fabsf(hi - lo) <= tol * (1.0f < amid ? amid : 1.0f)) {
            lo = hi = mid;
            break;
        }
        if (err > 0.0f) lo = mid; else hi = mid;
    }
    float theta = 0.5f * (lo + hi);
    for (int i = 0; i < n; ++i)
        out[i] = (s[i] > guard) ? sigmoid1((s[i] - theta) / temp) : 0.0f;
}

/* softmax_selected_scalar, :410-442 */
static void softmax_sel(const float* s, float* out, int n, float temp) {
    const float guard = -1.0e30f;
    for (int i = 0; i < n; ++i) out[i] = 0.0f;
    float mx = -INFINITY;
    for (int i = 0; i < n; ++i) {
        if (s[i] > guard) {
            float q = s[i] / temp;
            mx = (mx < q) ? q : mx;
        }
    }
    if (!isfinite(mx)) return;
    float sum = 0.0f;
    for (int i = 0; i < n; ++i) {
        if (s[i] > guard) {
            out[i] = safe_exp(s[i] / temp - mx);
            sum += out[i];
        }
    }
    if (!(sum > 0.0f) || !isfinite(sum)) {
        for (int i = 0; i < n; ++i) out[i] = 0.0f;
        return;
    }
    float inv = 1.0f / sum;
    for (int i = 0; i < n; ++i) out[i] *= inv;
}

/* decode_constrained, :1432-1672. The per-parent scan merges the reference's
 * fast scan (:476-509) and advanced scan (:512-549): both apply forced ->
 * banned -> min-EOS -> (n-gram) -> finite -> (repetition penalty) and insert
 * with raw = parent + lp, rank = raw * (1 / gnmt(len + 1)). */
int oracle_decode(const oracle_options* opt, const float* x, int T, int V,
                  const oracle_constraints* c, oracle_result* r) {
    if (!x) return fail("log_probs cannot be null");
    if (T <= 0) return fail("steps must be positive");
    if (V <= 0) return fail("vocab_size must be positive");
    if (opt->eos_token >= V) return fail("eos_token is outside vocab");
    if (c && c->forced_tokens) {
        for (int t = 0; t < T; ++t)
            if (c->forced_tokens[t] >= V) return fail("forced token is outside vocab");
    }
    if (opt->validate_inputs && validate(x, T, opt->beam_size, V)) return 1;

    const int min_len = (c && c->min_length >= 0) ? c->min_length : opt->min_length;
    const int K = opt->beam_size;
    const int P = oracle_pool_size(opt);
    const int eos = opt->eos_token;
    const float alpha = opt->length_penalty_alpha;
    const int advanced = c && (c->repetition_penalty > 1.0f || c->no_repeat_ngram_size > 0 || c->token_filter);
    const float log_pen = (c && c->repetition_penalty > 1.0f) ? logf(c->repetition_penalty) : 0.0f;

    for (size_t i = 0; i < (size_t)T * K; ++i) {
        r->parents[i] = -1; r->tokens[i] = -1; r->lengths[i] = 0;
        r->raw_scores[i] = -INFINITY; r->scores[i] = -INFINITY; r->weights[i] = 0.0f;
        r->from_logprob[i] = 0;
    }
    for (size_t i = 0; i < (size_t)T * P; ++i) {
        r->pool_parents[i] = -1; r->pool_tokens[i] = -1; r->pool_lengths[i] = 0;
        r->pool_raw_scores[i] = -INFINITY; r->pool_scores[i] = -INFINITY;
        r->relaxed_weights[i] = 0.0f; r->pool_from_logprob[i] = 0;
    }

    float* prev_raw = malloc(sizeof(float) * K);
    float* next_raw = malloc(sizeof(float) * K);
    int* prev_len = calloc(K, sizeof(int));
    int* next_len = calloc(K, sizeof(int));
    uint8_t* ended = calloc(K, 1);
    uint8_t* ended_next = calloc(K, 1);
    int32_t* seq = calloc((size_t)K * T, sizeof(int32_t));
    int32_t* seq_next = calloc((size_t)K * T, sizeof(int32_t));
    int* seq_len = calloc(K, sizeof(int));
    int* seq_len_next = calloc(K, sizeof(int));
    cand* top = malloc(sizeof(cand) * P);
    for (int k = 0; k < K; ++k) { prev_raw[k] = -INFINITY; next_raw[k] = -INFINITY; }
    prev_raw[0] = 0.0f;

    for (int t = 0; t < T; ++t) {
        for (int i = 0; i < P; ++i) {
            cand s = {-INFINITY, -INFINITY, -1, -1, 0, 0};
            top[i] = s;
        }
        const float* step = x + (size_t)t * K * V;
        const int forced = (c && c->forced_tokens) ? c->forced_tokens[t] : -1;
        for (int b = 0; b < K; ++b) {
            const float pr = prev_raw[b];
            if (!isfinite(pr)) continue;
            if (eos >= 0 && ended[b]) {
                int len = prev_len[b] < 1 ? 1 : prev_len[b];
                cand carry = {pr / gnmt(len, alpha), pr, b, eos, len, 0};
                push_top(top, P, &carry);
                continue;
            }
            const float* row = step + (size_t)b * V;
            const int new_len = prev_len[b] + 1;
            const float inv = 1.0f / gnmt(new_len, alpha);
            const int32_t* pre = seq + (size_t)b * T;
            const int plen = seq_len[b];
            for (int v = 0; v < V; ++v) {
                if (forced >= 0 && v != forced) continue;
                if (c && c->banned_tokens && c->banned_tokens[v]) continue;
                if (eos >= 0 && v == eos && new_len < min_len) continue;
                if (advanced && c->no_repeat_ngram_size > 0 &&
                    repeats_ngram(pre, plen, v, c->no_repeat_ngram_size)) continue;
                /* the filter sees the beam's prefix (NULL when empty) and runs
                 * after the n-gram check, before the finiteness check */
                if (advanced && c->token_filter &&
                    c->token_filter(c->token_filter_user_data, c->batch_index, t, b, plen ? pre : NULL, plen, v) == 0)
                    continue;
                float lp = row[v];
                if (!isfinite(lp)) continue;
                if (advanced && c->repetition_penalty > 1.0f && prefix_has(pre, plen, v))
                    lp = lp - log_pen;
                const float raw = pr + lp;
                const float rank = raw * inv;
                cand cd = {rank, raw, b, v, new_len, 1};
                push_top(top, P, &cd);
            }
        }
        for (int p = 0; p < P; ++p) {
            size_t i = (size_t)t * P + p;
            r->pool_parents[i] = top[p].parent;
            r->pool_tokens[i] = top[p].token;
            r->pool_lengths[i] = top[p].length;
            r->pool_raw_scores[i] = top[p].raw;
            r->pool_scores[i] = top[p].score;
            r->pool_from_logprob[i] = top[p].flp;
        }
        soft_topk(r->pool_scores + (size_t)t * P, r->relaxed_weights + (size_t)t * P, P, K,
                  opt->soft_topk_temperature, opt->soft_topk_tolerance, opt->soft_topk_max_iters);
        for (int k = 0; k < K; ++k) {
            size_t i = (size_t)t * K + k;
            r->parents[i] = top[k].parent;
            r->tokens[i] = top[k].token;
            r->lengths[i] = top[k].length;
            r->raw_scores[i] = top[k].raw;
            r->scores[i] = top[k].score;
            r->from_logprob[i] = top[k].flp;
            next_raw[k] = top[k].raw;
            next_len[k] = top[k].length;
            seq_len_next[k] = 0;
            if (top[k].parent >= 0) {
                int pb = top[k].parent;
                memcpy(seq_next + (size_t)k * T, seq + (size_t)pb * T, sizeof(int32_t) * seq_len[pb]);
                seq_len_next[k] = seq_len[pb];
                if (top[k].flp && top[k].token >= 0) seq_next[(size_t)k * T + seq_len_next[k]++] = top[k].token;
                ended_next[k] = (uint8_t)(ended[pb] || (eos >= 0 && top[k].token == eos));
            } else {
                ended_next[k] = 0;
            }
        }
        softmax_sel(r->scores + (size_t)t * K, r->weights + (size_t)t * K, K, opt->selected_temperature);
        for (int k = 0; k < K; ++k) {
            prev_raw[k] = next_raw[k]; next_raw[k] = -INFINITY;
            prev_len[k] = next_len[k]; next_len[k] = 0;
            ended[k] = ended_next[k]; ended_next[k] = 0;
            seq_len[k] = seq_len_next[k];
        }
        int32_t* tmp = seq; seq = seq_next; seq_next = tmp;
    }
    for (int k = 0; k < K; ++k) {
        r->final_raw_scores[k] = prev_raw[k];
        r->final_scores[k] = prev_raw[k] / gnmt(prev_len[k] < 1 ? 1 : prev_len[k], alpha);
    }
    free(prev_raw); free(next_raw); free(prev_len); free(next_len); free(ended);
    free(ended_next); free(seq); free(seq_next); free(seq_len); free(seq_len_next); free(top);
    return 0;
}

typedef struct entry { int64_t index; float value; } entry;

static int entry_cmp(const void* a, const void* b) {
    int64_t x = ((const entry*)a)->index, y = ((const entry*)b)->index;
    return (x > y) - (x < y);
}

/* Shared reverse sweep for the sparse and dense backward: backward_selected
 * (:1943-2003 / :2068-2124) then backward_relaxed_topk (:2005-2066 /
 * :2126-2186) per step, t = T-1 .. 0. Emits (index, draw) pairs through
 * either the entry list or the dense buffer. */
static void sweep(const oracle_options* opt, int T, int V, const oracle_result* f,
                  const float* gsel, const float* grel, const float* gfin,
                  entry* entries, int64_t* n_entries, float* dense, float* grad_initial) {
    const int K = opt->beam_size;
    const int P = oracle_pool_size(opt);
    const float alpha = opt->length_penalty_alpha;
    float* next = calloc(K, sizeof(float));
    float* prev = calloc(K, sizeof(float));
    int64_t n = 0;
#define EMIT(tt, parent, token, flp, draw)                                              \
    do {                                                                                \
        if ((parent) >= 0 && (draw) != 0.0f) {                                          \
            prev[(parent)] += (draw);                                                   \
            if ((flp) && (token) >= 0) {                                                \
                int64_t gi = ((int64_t)(tt) * K + (parent)) * (int64_t)V + (token);     \
                if (dense) dense[gi] += (draw);                                         \
                else { entries[n].index = gi; entries[n].value = (draw); ++n; }         \
            }                                                                           \
        }                                                                               \
    } while (0)
    for (int t = T - 1; t >= 0; --t) {
        for (int k = 0; k < K; ++k) prev[k] = 0.0f;
        const float* w = f->weights + (size_t)t * K;
        const float* gw = gsel ? gsel + (size_t)t * K : NULL;
        float dot = 0.0f;
        if (gw) for (int k = 0; k < K; ++k) dot += w[k] * gw[k];
        for (int k = 0; k < K; ++k) {
            size_t i = (size_t)t * K + k;
            int parent = f->parents[i];
            if (parent < 0) continue;
            float drank = 0.0f;
            if (gw) drank += (w[k] * (gw[k] - dot)) / opt->selected_temperature;
            if (gfin && t == T - 1) drank += gfin[k];
            int len = f->lengths[i] < 1 ? 1 : f->lengths[i];
            float inv = 1.0f / gnmt(len, alpha);
            float draw = next[k] + drank * inv;
            EMIT(t, parent, f->tokens[i], f->from_logprob[i], draw);
        }
        if (grel) {
            const float* rw = f->relaxed_weights + (size_t)t * P;
            const float* rg = grel + (size_t)t * P;
            float denom = 0.0f, numer = 0.0f;
            for (int p = 0; p < P; ++p) {
                float a = rw[p] * (1.0f - rw[p]);
                denom += a;
                numer += rg[p] * a;
            }
            if (denom > 1.0e-12f) {
                float center = numer / denom;
                float inv_temp = 1.0f / opt->soft_topk_temperature;
                for (int p = 0; p < P; ++p) {
                    size_t i = (size_t)t * P + p;
                    int parent = f->pool_parents[i];
                    if (parent < 0) continue;
                    float a = rw[p] * (1.0f - rw[p]);
                    float drank = a * inv_temp * (rg[p] - center);
                    if (drank == 0.0f) continue;
                    int len = f->pool_lengths[i] < 1 ? 1 : f->pool_lengths[i];
                    float inv = 1.0f / gnmt(len, alpha);
                    float draw = drank * inv;
                    EMIT(t, parent, f->pool_tokens[i], f->pool_from_logprob[i], draw);
                }
            }
        }
        float* tmp = next; next = prev; prev = tmp;
    }
#undef EMIT
    for (int k = 0; k < K; ++k) grad_initial[k] = next[k];
    if (n_entries) *n_entries = n;
    free(next); free(prev);
}

int oracle_backward_sparse(const oracle_options* opt, int T, int V, const oracle_result* f,
                           const float* gsel, const float* grel, const float* gfin,
                           int64_t* out_idx, float* out_val, int64_t* nnz, float* grad_initial) {
    const int K = opt->beam_size;
    const int P = oracle_pool_size(opt);
    entry* e = malloc(sizeof(entry) * ((size_t)T * (K + P) + 1));
    int64_t n = 0;
    sweep(opt, T, V, f, gsel, grel, gfin, e, &n, NULL, grad_initial);
    /* finalize_sparse_entries, :1908-1941: sort by index, sum duplicates. */
    qsort(e, (size_t)n, sizeof(entry), entry_cmp);
    int64_t m = 0;
    for (int64_t i = 0; i < n;) {
        int64_t j = i;
        float s = 0.0f;
        while (j < n && e[j].index == e[i].index) { s += e[j].value; ++j; }
        out_idx[m] = e[i].index;
        out_val[m] = s;
        ++m;
        i = j;
    }
    *nnz = m;
    free(e);
    return 0;
}

int oracle_backward_dense(const oracle_options* opt, int T, int V, const oracle_result* f,
                          const float* gsel, const float* grel, const float* gfin,
                          float* grad, float* grad_initial) {
    const int K = opt->beam_size;
    size_t count = (size_t)T * K * V;
    if ((long long)count > opt->max_dense_gradient_elements)
        return fail("dense gradient allocation exceeds max_dense_gradient_elements; use sparse backward");
    memset(grad, 0, count * sizeof(float));
    sweep(opt, T, V, f, gsel, grel, gfin, NULL, NULL, grad, grad_initial);
    return 0;
}
