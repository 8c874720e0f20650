/*
 * ORACLE - test infrastructure only (see eigen_restated.h).
 *
 * Restates src/eigen_engine.cpp step by step in C:
 *   load_bn           src/eigen_engine.cpp:52-67   BN fold, eps 1e-5
 *   architecture      src/eigen_engine.cpp:84-95
 *   im2col_3x3        src/eigen_engine.cpp:139-168 row ic*9+kh*3+kw, col oh*W+ow
 *   conv2d_3x3        src/eigen_engine.cpp:174-178 W[Cout, 9Cin] * col
 *   conv2d_1x1        src/eigen_engine.cpp:180-183
 *   batch_norm_apply  src/eigen_engine.cpp:185-190 x*scale + bias per row
 *   relu              src/eigen_engine.cpp:192-194
 *   linear            src/eigen_engine.cpp:196-199
 *   predict           src/eigen_engine.cpp:205-273
 * Matrices are stored row-major here ((rows, cols) element (r, c) at
 * r*cols + c); the only places where Eigen's column-major storage changes
 * the result are the input Map (:211) and the policy flatten (:242), which
 * ORC_LITERAL reproduces.
 */
#define _POSIX_C_SOURCE 200809L
#include "eigen_restated.h"

#include <math.h>
#include <pthread.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

typedef struct {
    char* name;
    int ndims;
    int64_t dims[8];
    float* data;
    int64_t count;
} orc_tensor;

typedef struct {
    float* w; /* [cout][cin*9] */
    int cout, cin;
    float* scale;
    float* bias;
} orc_conv;

struct orc_net {
    orc_tensor* t;
    int nt, cap;
    int ready;
    int board, hw, cin, filters, blocks, actions, hidden;
    orc_conv input;
    orc_conv* conv1;
    orc_conv* conv2;
    float *pconv_w, *pbn_s, *pbn_b, *pfc_w, *pfc_b;
    float *vconv_w, *vbn_s, *vbn_b, *v1_w, *v1_b, *v2_w, *v2_b;
};

orc_net* orc_new(void) { return (orc_net*)calloc(1, sizeof(orc_net)); }

static void free_conv(orc_conv* c) {
    free(c->scale);
    free(c->bias);
}

void orc_free(orc_net* net) {
    if (!net) return;
    for (int i = 0; i < net->nt; ++i) {
        free(net->t[i].name);
        free(net->t[i].data);
    }
    free(net->t);
    free_conv(&net->input);
    for (int b = 0; b < net->blocks && net->conv1; ++b) {
        free_conv(&net->conv1[b]);
        free_conv(&net->conv2[b]);
    }
    free(net->conv1);
    free(net->conv2);
    free(net->pbn_s);
    free(net->pbn_b);
    free(net->vbn_s);
    free(net->vbn_b);
    free(net);
}

int orc_set(orc_net* net, const char* name, const int64_t* dims, int ndims, const float* data) {
    if (!net || !name || ndims < 0 || ndims > 8) return -1;
    int64_t count = ndims > 0 ? 1 : 0;
    for (int i = 0; i < ndims; ++i) count *= dims[i];
    for (int i = 0; i < net->nt; ++i) {
        if (strcmp(net->t[i].name, name) == 0) { /* last one wins */
            free(net->t[i].data);
            net->t[i].data = NULL;
            net->t[i].ndims = ndims;
            memcpy(net->t[i].dims, dims, sizeof(int64_t) * (size_t)ndims);
            net->t[i].count = count;
            net->t[i].data = (float*)malloc(sizeof(float) * (size_t)(count > 0 ? count : 1));
            if (count > 0) memcpy(net->t[i].data, data, sizeof(float) * (size_t)count);
            net->ready = 0;
            return 0;
        }
    }
    if (net->nt == net->cap) {
        net->cap = net->cap ? 2 * net->cap : 64;
        net->t = (orc_tensor*)realloc(net->t, sizeof(orc_tensor) * (size_t)net->cap);
    }
    orc_tensor* t = &net->t[net->nt++];
    t->name = strdup(name);
    t->ndims = ndims;
    memcpy(t->dims, dims, sizeof(int64_t) * (size_t)ndims);
    t->count = count;
    t->data = (float*)malloc(sizeof(float) * (size_t)(count > 0 ? count : 1));
    if (count > 0) memcpy(t->data, data, sizeof(float) * (size_t)count);
    net->ready = 0;
    return 0;
}

static orc_tensor* find(orc_net* net, const char* name) {
    for (int i = 0; i < net->nt; ++i)
        if (strcmp(net->t[i].name, name) == 0) return &net->t[i];
    return NULL;
}

/* Fetches a tensor with an exact element count; records "Missing tensor: "
 * like src/eigen_engine.cpp:30. */
static float* need(orc_net* net, const char* name, int64_t count, char* err, int errlen) {
    orc_tensor* t = find(net, name);
    if (!t) {
        snprintf(err, (size_t)errlen, "Missing tensor: %s", name);
        return NULL;
    }
    if (t->count != count) {
        snprintf(err, (size_t)errlen, "Tensor %s has %lld values, expected %lld", name,
                 (long long)t->count, (long long)count);
        return NULL;
    }
    return t->data;
}

/* src/eigen_engine.cpp:52-67 */
static int load_bn(orc_net* net, const char* prefix, int ch, float** scale, float** bias,
                   char* err, int errlen) {
    char nm[256];
    snprintf(nm, sizeof nm, "%s.weight", prefix);
    float* g = need(net, nm, ch, err, errlen);
    snprintf(nm, sizeof nm, "%s.bias", prefix);
    float* b = need(net, nm, ch, err, errlen);
    snprintf(nm, sizeof nm, "%s.running_mean", prefix);
    float* m = need(net, nm, ch, err, errlen);
    snprintf(nm, sizeof nm, "%s.running_var", prefix);
    float* v = need(net, nm, ch, err, errlen);
    if (!g || !b || !m || !v) return -1;
    const float eps = 1e-5f;
    *scale = (float*)malloc(sizeof(float) * (size_t)ch);
    *bias = (float*)malloc(sizeof(float) * (size_t)ch);
    for (int i = 0; i < ch; ++i) {
        float inv_std = 1.0f / sqrtf(v[i] + eps);
        (*scale)[i] = g[i] * inv_std;
        (*bias)[i] = b[i] - g[i] * m[i] * inv_std;
    }
    return 0;
}

static int load_conv(orc_net* net, orc_conv* c, const char* wname, const char* bn, int cout,
                     int cin, char* err, int errlen) {
    c->cout = cout;
    c->cin = cin;
    c->w = need(net, wname, (int64_t)cout * cin * 9, err, errlen);
    if (!c->w) return -1;
    return load_bn(net, bn, cout, &c->scale, &c->bias, err, errlen);
}

int orc_finalize(orc_net* net, char* err, int errlen) {
    char nm[256];
    orc_tensor* iw = find(net, "input_conv.weight");
    if (!iw || iw->ndims != 4) {
        snprintf(err, (size_t)errlen, "Missing tensor: input_conv.weight");
        return -1;
    }
    net->cin = (int)iw->dims[1];
    net->filters = (int)iw->dims[0];
    net->blocks = 0;
    for (;;) {
        snprintf(nm, sizeof nm, "res_blocks.%d.conv1.weight", net->blocks);
        if (!find(net, nm)) break;
        net->blocks++;
    }
    orc_tensor* pw = find(net, "policy_fc.weight");
    if (!pw || pw->ndims != 2) {
        snprintf(err, (size_t)errlen, "Missing tensor: policy_fc.weight");
        return -1;
    }
    net->actions = (int)pw->dims[0];
    net->board = (int)sqrtf((float)(net->actions - 1));
    net->hw = net->board * net->board;
    const int C = net->filters, HW = net->hw, A = net->actions;
    if (load_conv(net, &net->input, "input_conv.weight", "input_bn", C, net->cin, err, errlen))
        return -1;
    net->conv1 = (orc_conv*)calloc((size_t)(net->blocks ? net->blocks : 1), sizeof(orc_conv));
    net->conv2 = (orc_conv*)calloc((size_t)(net->blocks ? net->blocks : 1), sizeof(orc_conv));
    for (int b = 0; b < net->blocks; ++b) {
        char w1[128], w2[128], b1[128], b2[128];
        snprintf(w1, sizeof w1, "res_blocks.%d.conv1.weight", b);
        snprintf(b1, sizeof b1, "res_blocks.%d.bn1", b);
        snprintf(w2, sizeof w2, "res_blocks.%d.conv2.weight", b);
        snprintf(b2, sizeof b2, "res_blocks.%d.bn2", b);
        if (load_conv(net, &net->conv1[b], w1, b1, C, C, err, errlen)) return -1;
        if (load_conv(net, &net->conv2[b], w2, b2, C, C, err, errlen)) return -1;
    }
    if (!(net->pconv_w = need(net, "policy_conv.weight", 2 * C, err, errlen))) return -1;
    if (load_bn(net, "policy_bn", 2, &net->pbn_s, &net->pbn_b, err, errlen)) return -1;
    if (!(net->pfc_w = need(net, "policy_fc.weight", (int64_t)A * 2 * HW, err, errlen))) return -1;
    if (!(net->pfc_b = need(net, "policy_fc.bias", A, err, errlen))) return -1;
    if (!(net->vconv_w = need(net, "value_conv.weight", C, err, errlen))) return -1;
    if (load_bn(net, "value_bn", 1, &net->vbn_s, &net->vbn_b, err, errlen)) return -1;
    orc_tensor* v1 = find(net, "value_fc1.weight");
    if (!v1 || v1->ndims != 2) {
        snprintf(err, (size_t)errlen, "Missing tensor: value_fc1.weight");
        return -1;
    }
    net->hidden = (int)v1->dims[0];
    const int H = net->hidden;
    if (!(net->v1_w = need(net, "value_fc1.weight", (int64_t)H * HW, err, errlen))) return -1;
    if (!(net->v1_b = need(net, "value_fc1.bias", H, err, errlen))) return -1;
    if (!(net->v2_w = need(net, "value_fc2.weight", H, err, errlen))) return -1;
    if (!(net->v2_b = need(net, "value_fc2.bias", 1, err, errlen))) return -1;
    net->ready = 1;
    return 0;
}

int orc_info(const orc_net* net, int* board, int* input_channels, int* filters, int* blocks,
             int* actions) {
    if (!net || !net->ready) return -1;
    if (board) *board = net->board;
    if (input_channels) *input_channels = net->cin;
    if (filters) *filters = net->filters;
    if (blocks) *blocks = net->blocks;
    if (actions) *actions = net->actions;
    return 0;
}

/* ---- forward ------------------------------------------------------------ */

typedef struct {
    float* col;   /* [9*Cmax][HW] */
    float* a;     /* [C][HW] trunk */
    float* b;     /* [C][HW] */
    float* c;     /* [C][HW] */
    float* x0;    /* [Cin][HW] */
    float* pflat; /* [2*HW] */
    float* vflat; /* [HW] */
    float* hid;   /* [H] */
    float* lg;    /* [A] */
} orc_scratch;

/* src/eigen_engine.cpp:139-168 */
static void im2col_3x3(const float* in, int cin, int h, int w, float* col) {
    const int hw = h * w;
    for (int ic = 0; ic < cin; ++ic)
        for (int kh = 0; kh < 3; ++kh)
            for (int kw = 0; kw < 3; ++kw) {
                float* row = col + (size_t)(ic * 9 + kh * 3 + kw) * hw;
                for (int oh = 0; oh < h; ++oh) {
                    const int ih = oh + kh - 1;
                    for (int ow = 0; ow < w; ++ow) {
                        const int iw = ow + kw - 1;
                        row[oh * w + ow] = (ih >= 0 && ih < h && iw >= 0 && iw < w)
                                               ? in[(size_t)ic * hw + ih * w + iw]
                                               : 0.0f;
                    }
                }
            }
}

/* out[co][p] = sum_k W[co][k] * col[k][p]  (src/eigen_engine.cpp:177).
 * Four output rows at a time so each col row is streamed once per group;
 * the p loop is contiguous and vectorises. */
static void gemm_rows(const float* W, int cout, int K, const float* col, int hw, float* out) {
    int co = 0;
    for (; co + 4 <= cout; co += 4) {
        float* o0 = out + (size_t)co * hw;
        float* o1 = o0 + hw;
        float* o2 = o1 + hw;
        float* o3 = o2 + hw;
        memset(o0, 0, sizeof(float) * (size_t)hw * 4);
        const float* w0 = W + (size_t)co * K;
        const float* w1 = w0 + K;
        const float* w2 = w1 + K;
        const float* w3 = w2 + K;
        for (int k = 0; k < K; ++k) {
            const float a0 = w0[k], a1 = w1[k], a2 = w2[k], a3 = w3[k];
            const float* cr = col + (size_t)k * hw;
            for (int p = 0; p < hw; ++p) {
                const float v = cr[p];
                o0[p] += a0 * v;
                o1[p] += a1 * v;
                o2[p] += a2 * v;
                o3[p] += a3 * v;
            }
        }
    }
    for (; co < cout; ++co) {
        float* o = out + (size_t)co * hw;
        memset(o, 0, sizeof(float) * (size_t)hw);
        const float* wr = W + (size_t)co * K;
        for (int k = 0; k < K; ++k) {
            const float a = wr[k];
            const float* cr = col + (size_t)k * hw;
            for (int p = 0; p < hw; ++p) o[p] += a * cr[p];
        }
    }
}

/* src/eigen_engine.cpp:185-190 */
static void bn_apply(float* x, int ch, int hw, const float* scale, const float* bias) {
    for (int c = 0; c < ch; ++c)
        for (int p = 0; p < hw; ++p) x[(size_t)c * hw + p] = x[(size_t)c * hw + p] * scale[c] + bias[c];
}

/* src/eigen_engine.cpp:192-194 */
static void relu(float* x, size_t n) {
    for (size_t i = 0; i < n; ++i) x[i] = x[i] > 0.0f ? x[i] : 0.0f;
}

static void conv_bn(const orc_net* net, const orc_conv* cv, const float* in, float* out,
                    orc_scratch* s) {
    im2col_3x3(in, cv->cin, net->board, net->board, s->col);
    gemm_rows(cv->w, cv->cout, cv->cin * 9, s->col, net->hw, out);
    bn_apply(out, cv->cout, net->hw, cv->scale, cv->bias);
}

/* src/eigen_engine.cpp:205-273 for one position. */
static void predict_one(const orc_net* net, const float* state, int mode, orc_scratch* s,
                        float* probs, float* logits, float* value) {
    const int C = net->filters, HW = net->hw, A = net->actions, H = net->hidden, Cin = net->cin;
    /* :211 - Map<const Tensor>(state, Cin, HW) */
    for (int c = 0; c < Cin; ++c)
        for (int p = 0; p < HW; ++p)
            s->x0[(size_t)c * HW + p] =
                mode == ORC_LITERAL ? state[c + (size_t)p * Cin] : state[(size_t)c * HW + p];
    /* :214-217 */
    conv_bn(net, &net->input, s->x0, s->a, s);
    relu(s->a, (size_t)C * HW);
    /* :220-234 */
    for (int b = 0; b < net->blocks; ++b) {
        conv_bn(net, &net->conv1[b], s->a, s->b, s);
        relu(s->b, (size_t)C * HW);
        conv_bn(net, &net->conv2[b], s->b, s->c, s);
        for (size_t i = 0; i < (size_t)C * HW; ++i) s->a[i] = s->c[i] + s->a[i];
        relu(s->a, (size_t)C * HW);
    }
    /* :237-242 policy 1x1 conv, BN, ReLU, flatten */
    float* pc = s->b; /* (2, HW) */
    gemm_rows(net->pconv_w, 2, C, s->a, HW, pc);
    bn_apply(pc, 2, HW, net->pbn_s, net->pbn_b);
    relu(pc, (size_t)2 * HW);
    for (int c = 0; c < 2; ++c)
        for (int p = 0; p < HW; ++p)
            s->pflat[mode == ORC_LITERAL ? (c + 2 * p) : (c * HW + p)] = pc[(size_t)c * HW + p];
    /* :243-244 */
    for (int a = 0; a < A; ++a) {
        const float* wr = net->pfc_w + (size_t)a * 2 * HW;
        float acc = 0.0f;
        for (int i = 0; i < 2 * HW; ++i) acc += wr[i] * s->pflat[i];
        s->lg[a] = acc + net->pfc_b[a];
    }
    /* :247-250 softmax */
    float mx = s->lg[0];
    for (int a = 1; a < A; ++a) mx = s->lg[a] > mx ? s->lg[a] : mx;
    float sum = 0.0f;
    for (int a = 0; a < A; ++a) sum += expf(s->lg[a] - mx);
    for (int a = 0; a < A; ++a) probs[a] = expf(s->lg[a] - mx) / sum;
    if (logits)
        for (int a = 0; a < A; ++a) logits[a] = s->lg[a];
    /* :257-269 value head */
    gemm_rows(net->vconv_w, 1, C, s->a, HW, s->vflat);
    bn_apply(s->vflat, 1, HW, net->vbn_s, net->vbn_b);
    relu(s->vflat, (size_t)HW);
    for (int j = 0; j < H; ++j) {
        const float* wr = net->v1_w + (size_t)j * HW;
        float acc = 0.0f;
        for (int p = 0; p < HW; ++p) acc += wr[p] * s->vflat[p];
        acc += net->v1_b[j];
        s->hid[j] = acc > 0.0f ? acc : 0.0f;
    }
    float v = 0.0f;
    for (int j = 0; j < H; ++j) v += net->v2_w[j] * s->hid[j];
    *value = tanhf(v + net->v2_b[0]);
}

static int scratch_init(const orc_net* net, orc_scratch* s) {
    const int C = net->filters, HW = net->hw;
    const int cmax = C > net->cin ? C : net->cin;
    memset(s, 0, sizeof *s);
    s->col = (float*)malloc(sizeof(float) * (size_t)9 * cmax * HW);
    s->a = (float*)malloc(sizeof(float) * (size_t)C * HW);
    s->b = (float*)malloc(sizeof(float) * (size_t)C * HW);
    s->c = (float*)malloc(sizeof(float) * (size_t)C * HW);
    s->x0 = (float*)malloc(sizeof(float) * (size_t)net->cin * HW);
    s->pflat = (float*)malloc(sizeof(float) * (size_t)2 * HW);
    s->vflat = (float*)malloc(sizeof(float) * (size_t)HW);
    s->hid = (float*)malloc(sizeof(float) * (size_t)(net->hidden > 0 ? net->hidden : 1));
    s->lg = (float*)malloc(sizeof(float) * (size_t)net->actions);
    return (s->col && s->a && s->b && s->c && s->x0 && s->pflat && s->vflat && s->hid && s->lg) ? 0
                                                                                                 : -1;
}

static void scratch_free(orc_scratch* s) {
    free(s->col);
    free(s->a);
    free(s->b);
    free(s->c);
    free(s->x0);
    free(s->pflat);
    free(s->vflat);
    free(s->hid);
    free(s->lg);
}

typedef struct {
    const orc_net* net;
    const float* states;
    int begin, end, mode;
    float *probs, *logits, *values;
    int rc;
} orc_job;

static void* run_job(void* arg) {
    orc_job* j = (orc_job*)arg;
    const orc_net* net = j->net;
    const size_t in_per = (size_t)net->cin * net->hw;
    orc_scratch s;
    if (scratch_init(net, &s)) {
        scratch_free(&s);
        j->rc = -1;
        return NULL;
    }
    for (int i = j->begin; i < j->end; ++i)
        predict_one(net, j->states + (size_t)i * in_per, j->mode, &s,
                    j->probs + (size_t)i * net->actions,
                    j->logits ? j->logits + (size_t)i * net->actions : NULL, j->values + i);
    scratch_free(&s);
    j->rc = 0;
    return NULL;
}

int orc_predict_batch(const orc_net* net, const float* states, int n, int mode, int threads,
                      float* probs, float* logits, float* values) {
    if (!net || !net->ready || n < 0) return -1;
    if (n == 0) return 0;
    if (threads < 1) threads = 1;
    if (threads > n) threads = n;
    orc_job* jobs = (orc_job*)calloc((size_t)threads, sizeof(orc_job));
    pthread_t* tids = (pthread_t*)calloc((size_t)threads, sizeof(pthread_t));
    int rc = 0;
    for (int t = 0; t < threads; ++t) {
        jobs[t].net = net;
        jobs[t].states = states;
        jobs[t].begin = (int)((long)n * t / threads);
        jobs[t].end = (int)((long)n * (t + 1) / threads);
        jobs[t].mode = mode;
        jobs[t].probs = probs;
        jobs[t].logits = logits;
        jobs[t].values = values;
    }
    if (threads == 1) {
        run_job(&jobs[0]);
        rc = jobs[0].rc;
    } else {
        for (int t = 0; t < threads; ++t) pthread_create(&tids[t], NULL, run_job, &jobs[t]);
        for (int t = 0; t < threads; ++t) {
            pthread_join(tids[t], NULL);
            if (jobs[t].rc) rc = -1;
        }
    }
    free(jobs);
    free(tids);
    return rc;
}
