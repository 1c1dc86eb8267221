/*
 * hf_oracle.c -- CPU restatement of HummingFlight's MoE layer (parity oracle).
 *
 * TEST INFRASTRUCTURE, never the product. See hf_oracle.h for the contract and
 * the reference lines each function follows. Built with -O3 -fopenmp
 * -ffp-contract=off (oracle/Makefile) so every fp32 operation is the single
 * rounded operation the reference performs.
 */
#include "hf_oracle.h"
#include "hf_gen.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

int hfo_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* compute/cpu_kernels.cpp:82-93. Eight rows advance together so the loop has
 * independent dependency chains; each row still sums j = 0..K-1 in order. */
void hfo_gemv_bf16_f32(const uint16_t* A, const float* x, float* y, int M, int K,
                       float alpha, float beta) {
    const int nblk = (M + 7) / 8;
#pragma omp parallel for schedule(static) if ((long long)M * K > (1 << 16))
    for (int b = 0; b < nblk; ++b) {
        const int r0 = b * 8;
        const int nr = (M - r0) < 8 ? (M - r0) : 8;
        float dot[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        const uint16_t* rows[8];
        for (int r = 0; r < 8; ++r) rows[r] = A + (int64_t)(r0 + (r < nr ? r : 0)) * K;
        for (int j = 0; j < K; ++j) {
            const float xj = x[j];
            for (int r = 0; r < 8; ++r) {
                float p = hfg_bf16_to_f32(rows[r][j]) * xj;
                dot[r] = dot[r] + p;
            }
        }
        for (int r = 0; r < nr; ++r) {
            float a = alpha * dot[r];
            float c = beta * y[r0 + r];
            y[r0 + r] = a + c;
        }
    }
}

/* model/glm_forward.cpp:519-524 */
void hfo_router_scores(const uint16_t* router_w, const float* x, int E, int H, float* scores) {
    hfo_gemv_bf16_f32(router_w, x, scores, E, H, 1.0f, 0.0f);
    for (int i = 0; i < E; ++i) scores[i] = 1.0f / (1.0f + expf(-scores[i]));
}

/* model/glm_forward.cpp:185-197 */
void hfo_rmsnorm(const float* x, const uint16_t* w, float eps, int n, float* out) {
    float sq = 0.0f;
    for (int i = 0; i < n; ++i) sq += x[i] * x[i];
    const float rms = 1.0f / sqrtf(sq / (float)n + eps);
    for (int i = 0; i < n; ++i) {
        const float v = x[i] * rms;
        out[i] = w ? v * hfg_bf16_to_f32(w[i]) : v;
    }
}

/* model/glm_forward.cpp:795-796: hiddenStates = residual; hiddenStates += mlpOut */
void hfo_residual_add(const float* x, const float* mlp_out, int n, float* out) {
    for (int i = 0; i < n; ++i) out[i] = x[i] + mlp_out[i];
}

/* compute/moe_router.h:29-57 (selection by repeated arg-max is the same set
 * and order as the descending partial_sort, with ties to the lower id). */
int hfo_topk_scores(const float* scores, int E, const float* bias, int top_k, float scale,
                    int norm, int32_t* idx, float* w, float* margin_out) {
    if (E <= 0 || top_k <= 0) {
        if (margin_out) *margin_out = INFINITY;
        return 0;
    }
    const int k = top_k < E ? top_k : E;
    float* adj = (float*)malloc(sizeof(float) * (size_t)E);
    unsigned char* taken = (unsigned char*)calloc((size_t)E, 1);
    for (int i = 0; i < E; ++i) adj[i] = scores[i] + (bias ? bias[i] : 0.0f);
    float kth = 0.0f;
    for (int s = 0; s < k; ++s) {
        int best = -1;
        for (int i = 0; i < E; ++i) {
            if (taken[i]) continue;
            if (best < 0 || adj[i] > adj[best]) best = i;
        }
        taken[best] = 1;
        idx[s] = best;
        kth = adj[best];
    }
    if (margin_out) {
        float next = -INFINITY;
        int found = 0;
        for (int i = 0; i < E; ++i)
            if (!taken[i] && (!found || adj[i] > next)) { next = adj[i]; found = 1; }
        *margin_out = found ? (kth - next) : INFINITY;
    }
    float sum = 0.0f;
    for (int i = 0; i < k; ++i) {
        w[i] = scores[idx[i]];
        sum += w[i];
    }
    if (norm && sum > 0.0f)
        for (int i = 0; i < k; ++i) w[i] /= sum;
    for (int i = 0; i < k; ++i) w[i] *= scale;
    free(adj);
    free(taken);
    return k;
}

/* model/glm_forward.cpp:434-449 (and :459-479 for the shared expert). */
void hfo_expert_ffn(const uint16_t* gate, const uint16_t* up, const uint16_t* down,
                    const float* x, float* y, int H, int I) {
    /* zero-filled like GLMForward::ensureFloat's vectors: gemv reads y (beta*y) */
    float* g = (float*)calloc((size_t)I, sizeof(float));
    float* u = (float*)calloc((size_t)I, sizeof(float));
    float* mid = (float*)calloc((size_t)I, sizeof(float));
    hfo_gemv_bf16_f32(gate, x, g, I, H, 1.0f, 0.0f);
    hfo_gemv_bf16_f32(up, x, u, I, H, 1.0f, 0.0f);
    for (int i = 0; i < I; ++i) mid[i] = g[i] / (1.0f + expf(-g[i])) * u[i];
    hfo_gemv_bf16_f32(down, mid, y, H, I, 1.0f, 0.0f);
    free(g);
    free(u);
    free(mid);
}

/* The scalar GEMV of compute/cpu_kernels.cpp:82-93 for n vectors at once:
 * yT[i*n + t] = alpha * dot(A[i,:], x_t) + beta * yT[i*n + t], with x given
 * transposed (xT[j*n + t]). Every (row, vector) pair still sums j = 0..K-1
 * in order with one rounded multiply and one rounded add per term, so each
 * result is bit-identical to hfo_gemv_bf16_f32 on that vector alone; only
 * the loop nest changes (four rows share each weight load, and the vectors
 * sit side by side so the token loop vectorises without reassociation). */
#define HFO_NB 16
static void gemv_multi(const uint16_t* A, const float* xT, int n, float* yT, int M, int K,
                       float alpha, float beta) {
    const int nrb = (M + 3) / 4;
#pragma omp parallel for schedule(static)
    for (int rb = 0; rb < nrb; ++rb) {
        const int r0 = rb * 4;
        const int nr = (M - r0) < 4 ? (M - r0) : 4;
        const uint16_t* rows[4];
        for (int r = 0; r < 4; ++r) rows[r] = A + (int64_t)(r0 + (r < nr ? r : 0)) * K;
        for (int t0 = 0; t0 < n; t0 += HFO_NB) {
            const int nt = (n - t0) < HFO_NB ? (n - t0) : HFO_NB;
            float acc[4][HFO_NB];
            for (int r = 0; r < 4; ++r)
                for (int t = 0; t < HFO_NB; ++t) acc[r][t] = 0.0f;
            for (int j = 0; j < K; ++j) {
                const float* xj = xT + (int64_t)j * n + t0;
                float xv[HFO_NB];
                for (int t = 0; t < HFO_NB; ++t) xv[t] = t < nt ? xj[t] : 0.0f;
                for (int r = 0; r < 4; ++r) {
                    const float w = hfg_bf16_to_f32(rows[r][j]);
                    for (int t = 0; t < HFO_NB; ++t) {
                        float p = w * xv[t];
                        acc[r][t] = acc[r][t] + p;
                    }
                }
            }
            for (int r = 0; r < nr; ++r)
                for (int t = 0; t < nt; ++t) {
                    float* y = yT + (int64_t)(r0 + r) * n + t0 + t;
                    float a = alpha * acc[r][t];
                    float c = beta * *y;
                    *y = a + c;
                }
        }
    }
}

/* expertFFNRaw (model/glm_forward.cpp:434-449) for n tokens of one expert:
 * x rows [n x H] -> y rows [n x H] (y is read for the beta * y term of the
 * down GEMV, as hfo_expert_ffn's zero-filled output is). Bit-identical per
 * token to hfo_expert_ffn. */
void hfo_expert_ffn_multi(const uint16_t* gate, const uint16_t* up, const uint16_t* down,
                          const float* x, float* y, int n, int H, int I) {
    if (n <= 0) return;
    float* xT = (float*)malloc(sizeof(float) * (size_t)H * n);
    float* g = (float*)calloc((size_t)I * n, sizeof(float));
    float* u = (float*)calloc((size_t)I * n, sizeof(float));
    float* yT = (float*)malloc(sizeof(float) * (size_t)H * n);
    for (int t = 0; t < n; ++t)
        for (int j = 0; j < H; ++j) xT[(size_t)j * n + t] = x[(size_t)t * H + j];
    gemv_multi(gate, xT, n, g, I, H, 1.0f, 0.0f);
    gemv_multi(up, xT, n, u, I, H, 1.0f, 0.0f);
    /* mid = g / (1 + exp(-g)) * u in fp32, laid out [I x n] for the down GEMV */
    for (size_t i = 0; i < (size_t)I * n; ++i) g[i] = g[i] / (1.0f + expf(-g[i])) * u[i];
    for (int t = 0; t < n; ++t)
        for (int h = 0; h < H; ++h) yT[(size_t)h * n + t] = y[(size_t)t * H + h];
    gemv_multi(down, g, n, yT, H, I, 1.0f, 0.0f);
    for (int t = 0; t < n; ++t)
        for (int h = 0; h < H; ++h) y[(size_t)t * H + h] = yT[(size_t)h * n + t];
    free(xT);
    free(g);
    free(u);
    free(yT);
}

void hfo_permute(const int32_t* ids, int T, int k, int E, int has_shared, int32_t* counts,
                 int32_t* offsets, int32_t* perm) {
    for (int e = 0; e <= E; ++e) counts[e] = 0;
    for (int s = 0; s < T * k; ++s) counts[ids[s]]++;
    counts[E] = has_shared ? T : 0;
    offsets[0] = 0;
    for (int e = 0; e <= E; ++e) offsets[e + 1] = offsets[e] + counts[e];
    int32_t* cur = (int32_t*)malloc(sizeof(int32_t) * (size_t)(E + 1));
    memcpy(cur, offsets, sizeof(int32_t) * (size_t)(E + 1));
    for (int t = 0; t < T; ++t)        /* token-major scan keeps token order */
        for (int i = 0; i < k; ++i) {
            const int e = ids[t * k + i];
            perm[cur[e]++] = t * k + i;
        }
    if (has_shared)
        for (int t = 0; t < T; ++t) perm[cur[E]++] = T * k + t;
    free(cur);
}

/* Router + top-k for every token (glm_forward.cpp:517-541). The router
 * GEMV runs for up to 512 tokens at a time through gemv_multi (per token the
 * same sums as hfo_router_scores), then sigmoid and topKScores per token. */
static void route_all(const hfo_dims* d, const uint16_t* router_w, const float* bias,
                      const float* x, int T, int32_t* ids, float* w, float* margins) {
    const int E = d->num_experts, H = d->hidden;
    const int k = d->top_k < E ? d->top_k : E; /* TopKResult::k (moe_router.h:43) */
    const int CH = 512;
    float* scores = (float*)calloc((size_t)E, sizeof(float));
    float* xT = (float*)malloc(sizeof(float) * (size_t)H * CH);
    float* sT = (float*)malloc(sizeof(float) * (size_t)E * CH);
    for (int t0 = 0; t0 < T; t0 += CH) {
        const int n = (T - t0) < CH ? (T - t0) : CH;
        for (int t = 0; t < n; ++t)
            for (int j = 0; j < H; ++j) xT[(size_t)j * n + t] = x[(size_t)(t0 + t) * H + j];
        for (size_t i = 0; i < (size_t)E * n; ++i) sT[i] = 0.0f;
        gemv_multi(router_w, xT, n, sT, E, H, 1.0f, 0.0f);
        for (int t = 0; t < n; ++t) {
            for (int e = 0; e < E; ++e) scores[e] = 1.0f / (1.0f + expf(-sT[(size_t)e * n + t]));
            float m;
            hfo_topk_scores(scores, E, bias, k, d->scale, d->norm_topk,
                            ids + (size_t)(t0 + t) * k, w + (size_t)(t0 + t) * k, &m);
            if (margins) margins[t0 + t] = m;
        }
    }
    free(scores);
    free(xT);
    free(sT);
}

/* Expert FFN for every token routed to one expert, into slot_out rows
 * (one batched pass over the expert's weights; per token the same
 * arithmetic as hfo_expert_ffn). */
static void run_expert(const hfo_dims* d, const uint16_t* gud, int I, const float* x,
                       int ntok, const int32_t* toks, const int32_t* slots, float* slot_out) {
    const int H = d->hidden;
    const uint16_t* g = gud;
    const uint16_t* u = gud + (size_t)I * H;
    const uint16_t* dn = u + (size_t)I * H;
    if (ntok <= 0) return;
    float* xs = (float*)malloc(sizeof(float) * (size_t)ntok * H);
    float* ys = (float*)malloc(sizeof(float) * (size_t)ntok * H);
    for (int j = 0; j < ntok; ++j) {
        memcpy(xs + (size_t)j * H, x + (size_t)toks[j] * H, sizeof(float) * (size_t)H);
        memcpy(ys + (size_t)j * H, slot_out + (size_t)slots[j] * H, sizeof(float) * (size_t)H);
    }
    hfo_expert_ffn_multi(g, u, dn, xs, ys, ntok, H, I);
    for (int j = 0; j < ntok; ++j)
        memcpy(slot_out + (size_t)slots[j] * H, ys + (size_t)j * H, sizeof(float) * (size_t)H);
    free(xs);
    free(ys);
}

/* Weighted accumulate in top-k rank order, then + shared
 * (glm_forward.cpp:555-556, 639-640, 658-660). */
static void combine(const hfo_dims* d, int T, int k, const float* w, const float* slot_out,
                    float* out) {
    const int H = d->hidden;
    for (int t = 0; t < T; ++t) {
        float* o = out + (size_t)t * H;
        for (int j = 0; j < H; ++j) o[j] = 0.0f;
        for (int i = 0; i < k; ++i) {
            const float wi = w[(size_t)t * k + i];
            const float* y = slot_out + ((size_t)t * k + i) * H;
            for (int j = 0; j < H; ++j) {
                float p = wi * y[j];
                o[j] = o[j] + p;
            }
        }
        if (d->shared_inter > 0) {
            const float* s = slot_out + ((size_t)T * k + t) * H;
            for (int j = 0; j < H; ++j) o[j] = o[j] + s[j];
        } else {
            for (int j = 0; j < H; ++j) o[j] = o[j] + 0.0f;
        }
    }
}

static int moe_common(const hfo_dims* d, const uint16_t* router_w, const float* bias,
                      const uint16_t* const* experts, const uint16_t* shared, uint64_t wseed,
                      uint32_t layer, const float* x, int T, float* out, int32_t* ids, float* w,
                      float* margins, float* slot_out) {
    const int E = d->num_experts, H = d->hidden;
    if (E <= 0 || d->top_k <= 0 || d->top_k > 8 || H <= 0 || T < 0) return 1;
    const int k = d->top_k < E ? d->top_k : E;
    if (T == 0) return 0;
    route_all(d, router_w, bias, x, T, ids, w, margins);

    const int has_shared = d->shared_inter > 0;
    int32_t* counts = (int32_t*)malloc(sizeof(int32_t) * (size_t)(E + 1));
    int32_t* offsets = (int32_t*)malloc(sizeof(int32_t) * (size_t)(E + 2));
    int32_t* perm = (int32_t*)malloc(sizeof(int32_t) * (size_t)(T * k + T));
    hfo_permute(ids, T, k, E, has_shared, counts, offsets, perm);

    float* slots = slot_out;
    if (!slots) slots = (float*)calloc((size_t)(T * k + T) * H, sizeof(float));
    int32_t* toks = (int32_t*)malloc(sizeof(int32_t) * (size_t)T);
    int32_t* sl = (int32_t*)malloc(sizeof(int32_t) * (size_t)T);
    uint16_t* buf = NULL;
    size_t maxI = (size_t)(d->inter > d->shared_inter ? d->inter : d->shared_inter);
    if (!experts) buf = (uint16_t*)malloc(sizeof(uint16_t) * 3 * maxI * (size_t)H);

    for (int e = 0; e <= E; ++e) {
        const int n = counts[e];
        if (n == 0) continue;
        const int I = (e == E) ? d->shared_inter : d->inter;
        for (int j = 0; j < n; ++j) {
            const int s = perm[offsets[e] + j];
            sl[j] = s;
            toks[j] = (e == E) ? (s - T * k) : (s / k);
        }
        const uint16_t* gud;
        if (experts) {
            gud = (e == E) ? shared : experts[e];
        } else {
            hfo_gen_expert(wseed, layer, (uint32_t)e, H, I, buf);
            gud = buf;
        }
        run_expert(d, gud, I, x, n, toks, sl, slots);
    }
    combine(d, T, k, w, slots, out);

    free(counts);
    free(offsets);
    free(perm);
    free(toks);
    free(sl);
    free(buf);
    if (!slot_out) free(slots);
    return 0;
}

int hfo_moe_layer(const hfo_dims* d, const uint16_t* router_w, const float* bias,
                  const uint16_t* const* experts, const uint16_t* shared, const float* x,
                  int T, float* out, int32_t* ids, float* w, float* margins, float* slot_out) {
    if (!experts || (d->shared_inter > 0 && !shared)) return 1;
    return moe_common(d, router_w, bias, experts, shared, 0, 0, x, T, out, ids, w, margins,
                      slot_out);
}

int hfo_moe_layer_synth(const hfo_dims* d, uint64_t wseed, uint32_t layer,
                        const float* bias_override, const float* x, int T, float* out,
                        int32_t* ids, float* w, float* margins, float* slot_out) {
    const int E = d->num_experts, H = d->hidden;
    uint16_t* router = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)E * H);
    float* bias = (float*)malloc(sizeof(float) * (size_t)E);
    hfo_gen_bf16_normal(wseed, layer, HFG_KIND_ROUTER, 0, 0.02, (uint64_t)E * H, router);
    if (bias_override)
        memcpy(bias, bias_override, sizeof(float) * (size_t)E);
    else
        hfo_gen_f32_uniform(wseed, layer, HFG_KIND_BIAS, 0, -0.1f, 0.1f, (uint64_t)E, bias);
    int rc = moe_common(d, router, bias, NULL, NULL, wseed, layer, x, T, out, ids, w, margins,
                        slot_out);
    free(router);
    free(bias);
    return rc;
}

void hfo_gen_bf16_normal(uint64_t seed, uint32_t layer, uint32_t kind, uint32_t expert,
                         double sigma, uint64_t n, uint16_t* out) {
    const uint64_t key = hfg_key(seed, layer, kind, expert);
    const float sc = hfg_normal_scale(sigma);
#pragma omp parallel for schedule(static) if (n > (1u << 20))
    for (int64_t i = 0; i < (int64_t)n; ++i)
        out[i] = hfg_f32_to_bf16(hfg_normal(key, (uint64_t)i, sc));
}

void hfo_gen_f32_uniform(uint64_t seed, uint32_t layer, uint32_t kind, uint32_t expert,
                         float lo, float hi, uint64_t n, float* out) {
    const uint64_t key = hfg_key(seed, layer, kind, expert);
    for (uint64_t i = 0; i < n; ++i) out[i] = hfg_uniform(key, i, lo, hi);
}

void hfo_gen_expert(uint64_t seed, uint32_t layer, uint32_t expert, int H, int I, uint16_t* out) {
    const uint64_t n = (uint64_t)H * (uint64_t)I;
    hfo_gen_bf16_normal(seed, layer, HFG_KIND_GATE, expert, 0.02, n, out);
    hfo_gen_bf16_normal(seed, layer, HFG_KIND_UP, expert, 0.02, n, out + n);
    hfo_gen_bf16_normal(seed, layer, HFG_KIND_DOWN, expert, 0.02, n, out + 2 * n);
}
