/*
 * CPU oracle for the torch-pyodide tensor-op hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker: a plain-C restatement of
 * the per-invocation arithmetic of the reference WGSL compute shaders
 * (the .wgsl files under runtime/src/vendor/torchjs/shaders) and of the host-side parameter
 * packing in the runtime/src/ops TypeScript files.  Only tests/, __graft_entry__.smoke() and
 * bench.py's CPU-baseline / reference arm may load it.  The CUDA product path
 * (libtpcuda.so) never links or calls it.
 *
 * Rules followed by every function:
 *   - f32 storage and f32 accumulators, in the shader's own loop order;
 *   - one C loop iteration per shader invocation (global_invocation_id.x), so
 *     the OpenMP parallel-for changes nothing in the result;
 *   - the 2-D dispatch bug of the reference (dispatch.ts:139-156, elements at
 *     and beyond x*256 never touched when a dispatch exceeds 65535 workgroups)
 *     is NOT restated: the oracle gives the per-invocation math the shader
 *     intends, at every size;
 *   - transcendental functions come from the host libm (expf, logf, sqrtf,
 *     cosf); WGSL allows several ulp there, so results are compared with a
 *     tolerance, never bit-for-bit, for anything that calls them.
 *
 * Build: gcc -O2 -fopenmp -ffp-contract=off -fPIC -shared (oracle/Makefile).
 * -ffp-contract=off keeps every a*b+c as two roundings, as the WGSL source
 * writes it.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>
#include <stdlib.h>

#define OR_EXPORT __attribute__((visibility("default")))

/* ------------------------------------------------------------------------- */
/* fill.wgsl:9-16                                                             */
OR_EXPORT void or_fill(float *out, int64_t n, float value) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) out[i] = value;
}

/* ------------------------------------------------------------------------- */
/* random.wgsl:11-21 xorshift / uint_to_float                                */
static inline uint32_t or_xorshift(uint32_t x) {
    x ^= x << 13;
    x ^= x >> 17;
    x ^= x << 5;
    return x;
}
static inline float or_u2f(uint32_t x) { return (float)x / 4294967296.0f; }

/* random.wgsl:23-48 (rand, randn), :50-65 normal_sample.  kind: 0 rand,
 * 1 randn, 2 normal(p0 mean, p1 std), 3 bernoulli(p0), 4 exponential(p0). */
OR_EXPORT void or_random(float *out, int64_t n, uint32_t seed, int kind, float p0, float p1) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) {
        uint32_t idx = (uint32_t)i;
        uint32_t s1 = or_xorshift(seed ^ (idx * 1664525u + 1013904223u));
        if (kind == 0) {
            out[i] = or_u2f(s1);
        } else if (kind == 1 || kind == 2) {
            uint32_t s2 = or_xorshift(s1);
            float u1 = or_u2f(s1), u2 = or_u2f(s2);
            float r = sqrtf(-2.0f * logf(fmaxf(u1, 0.0000001f)));
            float theta = 6.283185307179586f * u2;
            float z = r * cosf(theta);
            out[i] = (kind == 1) ? z : p0 + p1 * z;
        } else if (kind == 3) {
            out[i] = or_u2f(s1) < p0 ? 1.0f : 0.0f;
        } else {
            float u = fmaxf(or_u2f(s1), 1e-7f);
            out[i] = -logf(u) / p0;
        }
    }
}

/* ------------------------------------------------------------------------- */
/* elementwise.wgsl:5-31 (add/sub/mul/div_op), :85-114 (integer_pow, pow_op)  */
static float or_integer_pow(float base, float exponent) {
    float rounded = floorf(exponent + 0.5f);
    int n = (int)fabsf(rounded);
    float acc = 1.0f, factor = base;
    while (n > 0) {
        if ((n % 2) == 1) acc = acc * factor;
        factor = factor * factor;
        n = n / 2;
    }
    if (rounded < 0.0f) return 1.0f / acc;
    return acc;
}

static inline float or_binop(int op, float a, float b) {
    switch (op) {
    case 0: return a + b;
    case 1: return a - b;
    case 2: return a * b;
    case 3: return a / b;
    case 4: {
        float rounded = floorf(b + 0.5f);
        if (fabsf(b - rounded) < 0.000001f && fabsf(rounded) <= 64.0f) return or_integer_pow(a, b);
        return powf(a, b);
    }
    case 5: return fmaxf(a, b);               /* compare.wgsl maximum_op */
    case 6: return fminf(a, b);               /* compare.wgsl minimum_op */
    /* compare.wgsl:8-55: eq ne lt le gt ge -> 1.0 / 0.0 */
    case 10: return a == b ? 1.0f : 0.0f;
    case 11: return a != b ? 1.0f : 0.0f;
    case 12: return a < b ? 1.0f : 0.0f;
    case 13: return a <= b ? 1.0f : 0.0f;
    case 14: return a > b ? 1.0f : 0.0f;
    case 15: return a >= b ? 1.0f : 0.0f;
    default: return NAN;
    }
}

/* Broadcast binary op.  The reference first materialises each operand with
 * expand_broadcast.wgsl (broadcastOps.ts:84-111, index mapping :17-31) and
 * then runs the same-shape entry point.  The copy is exact, so the oracle maps
 * each output index straight to its source indices.  Shapes are right-aligned
 * (broadcastOps.ts:70-82); a_shape/b_shape are already padded to out ndim. */
OR_EXPORT void or_binary_bcast(int op, const float *a, const int64_t *a_shape, const float *b,
                               const int64_t *b_shape, float *out, const int64_t *out_shape, int ndim) {
    int64_t total = 1;
    for (int d = 0; d < ndim; ++d) total *= out_shape[d];
    int64_t as[8], bs[8];
    int64_t ra = 1, rb = 1;
    for (int d = ndim - 1; d >= 0; --d) {
        as[d] = a_shape[d] == 1 ? 0 : ra;
        bs[d] = b_shape[d] == 1 ? 0 : rb;
        ra *= a_shape[d];
        rb *= b_shape[d];
    }
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < total; ++i) {
        int64_t rem = i, ia = 0, ib = 0;
        for (int d = ndim - 1; d >= 0; --d) {
            int64_t c = rem % out_shape[d];
            rem /= out_shape[d];
            ia += c * as[d];
            ib += c * bs[d];
        }
        out[i] = or_binop(op, a[ia], b[ib]);
    }
}

/* ------------------------------------------------------------------------- */
/* unary.wgsl: neg :4-9, abs :11-16, sqrt :18-23, exp :25-30, log :39-44,
 * relu :81-86 (max(0,x)), reciprocal :206-210, rsqrt :213-217 (inverseSqrt),
 * square :220-225, sigmoid :74-79, tanh :67-72.                              */
static inline float or_unop(int op, float x) {
    switch (op) {
    case 0: return -x;
    case 1: return fabsf(x);
    case 2: return sqrtf(x);
    case 3: return expf(x);
    case 4: return logf(x);
    case 5: return fmaxf(0.0f, x);
    case 6: return 1.0f / sqrtf(x);
    case 7: return 1.0f / x;
    case 8: return x * x;
    case 9: return 1.0f / (1.0f + expf(-x));
    case 10: return tanhf(x);
    default: return NAN;
    }
}

OR_EXPORT void or_unary(int op, const float *in, float *out, int64_t n) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) out[i] = or_unop(op, in[i]);
}

/* arithmeticOps.ts:206-219 mulScalar: elementwise.wgsl mul with a one-element
 * operand buffer.  The shader indexes b[idx]; the scalar buffer is allocated at
 * full length and only word 0 is written, so only idx 0 sees the value in the
 * reference (a defect); the intended semantics x*value is restated here.       */
OR_EXPORT void or_mul_scalar(const float *in, float value, float *out, int64_t n) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) out[i] = in[i] * value;
}

/* ------------------------------------------------------------------------- */
/* transpose.wgsl transpose_2d (shapeOps.ts:715-725)                          */
OR_EXPORT void or_transpose2d(const float *in, float *out, int64_t rows, int64_t cols) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < rows * cols; ++i) {
        int64_t r = i / cols, c = i % cols;
        out[c * rows + r] = in[i];
    }
}

/* permute_nd.wgsl main (shapeOps.ts:125-154): out[j-coords] = in[coords with
 * source dim dims[j] = out coord j].                                         */
OR_EXPORT void or_permute(const float *in, const int64_t *in_shape, const int *dims, int ndim, float *out) {
    int64_t in_str[8], out_shape[8], total = 1;
    int64_t r = 1;
    for (int d = ndim - 1; d >= 0; --d) { in_str[d] = r; r *= in_shape[d]; }
    for (int d = 0; d < ndim; ++d) { out_shape[d] = in_shape[dims[d]]; total *= out_shape[d]; }
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < total; ++i) {
        int64_t rem = i, src = 0;
        for (int d = ndim - 1; d >= 0; --d) {
            int64_t c = rem % out_shape[d];
            rem /= out_shape[d];
            src += c * in_str[dims[d]];
        }
        out[i] = in[src];
    }
}

/* expand_broadcast.wgsl main (shapeOps.ts:305-329): in_shape padded to ndim. */
OR_EXPORT void or_expand(const float *in, const int64_t *in_shape, float *out, const int64_t *out_shape, int ndim) {
    int64_t st[8], r = 1, total = 1;
    for (int d = ndim - 1; d >= 0; --d) { st[d] = in_shape[d] == 1 ? 0 : r; r *= in_shape[d]; }
    for (int d = 0; d < ndim; ++d) total *= out_shape[d];
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < total; ++i) {
        int64_t rem = i, src = 0;
        for (int d = ndim - 1; d >= 0; --d) {
            int64_t c = rem % out_shape[d];
            rem /= out_shape[d];
            src += c * st[d];
        }
        out[i] = in[src];
    }
}

/* ------------------------------------------------------------------------- */
/* matmul.wgsl:52-66 matmul_2d and :68-85 matmul_3d: one output per
 * invocation, sequential k, f32 sum starting at 0.  batch = 1 gives 2-D.     */
OR_EXPORT void or_matmul(const float *A, const float *B, float *C, int64_t batch, int64_t M, int64_t K,
                         int64_t N, int b_batched) {
#pragma omp parallel for schedule(static)
    for (int64_t idx = 0; idx < batch * M * N; ++idx) {
        int64_t n = idx % N, m = (idx / N) % M, b = idx / (N * M);
        const float *a = A + (b * M + m) * K;
        const float *bb = B + (b_batched ? b * K * N : 0);
        float sum = 0.0f;
        for (int64_t k = 0; k < K; ++k) sum += a[k] * bb[k * N + n];
        C[idx] = sum;
    }
}

/* ------------------------------------------------------------------------- */
/* reduce_sum.wgsl / reduce_max.wgsl main + the host loop of
 * reductionOps.ts:161-213 reduceAll: repeated 256-wide workgroup trees until
 * one value is left, padding lanes with 0 (sum) or -1e38 (max).  mode 0 sum,
 * 1 mean (f32 sum read back, divided in f64 by the element count, stored as
 * f32: reductionOps.ts:203-210), 2 max.                                      */
OR_EXPORT float or_reduce_all(const float *in, int64_t n, int mode) {
    if (n <= 0) return mode == 2 ? -1.0e38f : 0.0f;
    float *cur = (float *)malloc(sizeof(float) * (size_t)n);
    memcpy(cur, in, sizeof(float) * (size_t)n);
    int64_t len = n;
    while (len > 1) {
        int64_t groups = (len + 255) / 256;
        float *nxt = (float *)malloc(sizeof(float) * (size_t)groups);
#pragma omp parallel for schedule(static)
        for (int64_t g = 0; g < groups; ++g) {
            float s[256];
            for (int l = 0; l < 256; ++l) {
                int64_t idx = g * 256 + l;
                s[l] = idx < len ? cur[idx] : (mode == 2 ? -1.0e38f : 0.0f);
            }
            for (int stride = 128; stride > 0; stride >>= 1)
                for (int l = 0; l < stride; ++l)
                    s[l] = (mode == 2) ? fmaxf(s[l], s[l + stride]) : s[l] + s[l + stride];
            nxt[g] = s[0];
        }
        free(cur);
        cur = nxt;
        len = groups;
    }
    float v = cur[0];
    free(cur);
    if (mode == 1) v = (float)((double)v / (double)n);
    return v;
}

/* reduce_dim.wgsl:12-63 (reductionOps.ts:215-251): one output per invocation,
 * sequential r.  op 0 sum, 1 mean (acc / f32(reduce)), 2 max (init -1e38).  */
OR_EXPORT void or_reduce_dim(const float *in, float *out, int64_t outer, int64_t reduce, int64_t inner, int op) {
#pragma omp parallel for schedule(static)
    for (int64_t o = 0; o < outer * inner; ++o) {
        int64_t b = o / inner, i = o % inner;
        float acc = (op == 2) ? -1e38f : 0.0f;
        const float *base = in + b * reduce * inner + i;
        for (int64_t r = 0; r < reduce; ++r) {
            float v = base[r * inner];
            if (op == 2) acc = fmaxf(acc, v); else acc += v;
        }
        out[o] = (op == 1) ? acc / (float)reduce : acc;
    }
}

/* argmax.wgsl:7-32: first index of the maximum (strict >), last dim.
 * Written as an index; the reference stores it as f32 with dtype int32.      */
OR_EXPORT void or_argmax(const float *in, int32_t *out, int64_t rows, int64_t n) {
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; ++r) {
        const float *x = in + r * n;
        float best = x[0];
        int32_t bi = 0;
        for (int64_t i = 1; i < n; ++i)
            if (x[i] > best) { best = x[i]; bi = (int32_t)i; }
        out[r] = bi;
    }
}

/* Max along a dim with the first-index tie-break: reduce_dim.wgsl op 2 for the
 * value (:28-30,45-46) and argmax.wgsl's strict > for the index (:23-28).
 * The reference itself routes max(dim) through sort (tensor_ops.py:1531-1537);
 * this is the intended result of that path.                                  */
OR_EXPORT void or_max_dim(const float *in, float *vals, int32_t *idx, int64_t outer, int64_t reduce, int64_t inner) {
#pragma omp parallel for schedule(static)
    for (int64_t o = 0; o < outer * inner; ++o) {
        int64_t b = o / inner, i = o % inner;
        const float *base = in + b * reduce * inner + i;
        float best = base[0];
        int32_t bi = 0;
        for (int64_t r = 1; r < reduce; ++r)
            if (base[r * inner] > best) { best = base[r * inner]; bi = (int32_t)r; }
        vals[o] = best;
        idx[o] = bi;
    }
}

/* softmax.wgsl:13-52: per row, max (strict >), sum exp(x-max), then
 * exp(x-max)/sum; rows = outer*inner, stride `inner` along the axis.         */
OR_EXPORT void or_softmax(const float *in, float *out, int64_t rows, int64_t axis, int64_t inner) {
#pragma omp parallel for schedule(static)
    for (int64_t row = 0; row < rows; ++row) {
        int64_t base = (row / inner) * axis * inner + (row % inner);
        float maxv = in[base];
        for (int64_t c = 1; c < axis; ++c) { float v = in[base + c * inner]; if (v > maxv) maxv = v; }
        float s = 0.0f;
        for (int64_t c = 0; c < axis; ++c) s = s + expf(in[base + c * inner] - maxv);
        for (int64_t c = 0; c < axis; ++c) out[base + c * inner] = expf(in[base + c * inner] - maxv) / s;
    }
}

/* log_softmax.wgsl:8-36 (reductionOps.ts:357-388; the host passes
 * batch = outer*inner and indexes rows as contiguous, i.e. last-dim only).   */
OR_EXPORT void or_log_softmax(const float *in, float *out, int64_t rows, int64_t C) {
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; ++r) {
        const float *x = in + r * C;
        float m = x[0];
        for (int64_t i = 1; i < C; ++i) m = fmaxf(m, x[i]);
        float s = 0.0f;
        for (int64_t i = 0; i < C; ++i) s += expf(x[i] - m);
        float lse = logf(s);
        for (int64_t i = 0; i < C; ++i) out[r * C + i] = x[i] - m - lse;
    }
}

/* softmax_backward.wgsl:17-35: gi = s * (go - sum_k go*s)                   */
OR_EXPORT void or_softmax_backward(const float *go, const float *s, float *gi, int64_t rows, int64_t C) {
#pragma omp parallel for schedule(static)
    for (int64_t idx = 0; idx < rows * C; ++idx) {
        int64_t row = idx / C;
        float dot = 0.0f;
        for (int64_t k = 0; k < C; ++k) dot = dot + go[row * C + k] * s[row * C + k];
        gi[idx] = s[idx] * (go[idx] - dot);
    }
}

/* log_softmax_backward.wgsl:17-34: gi = go - softmax * sum_k go             */
OR_EXPORT void or_log_softmax_backward(const float *go, const float *s, float *gi, int64_t rows, int64_t C) {
#pragma omp parallel for schedule(static)
    for (int64_t idx = 0; idx < rows * C; ++idx) {
        int64_t i = idx / C;
        float gs = 0.0f;
        for (int64_t k = 0; k < C; ++k) gs += go[i * C + k];
        gi[idx] = go[idx] - s[idx] * gs;
    }
}

/* cross_entropy.wgsl:9-39: per row logsumexp - logit[target], target read as
 * f32, cast with i32(), clamped to [0, C-1].                                 */
static inline uint32_t or_ce_target(float t, int64_t C) {
    int32_t ti = (int32_t)t;
    uint32_t u = (uint32_t)(ti > 0 ? ti : 0);
    return u < (uint32_t)(C - 1) ? u : (uint32_t)(C - 1);
}

OR_EXPORT void or_cross_entropy(const float *logits, const float *targets, float *loss, int64_t B, int64_t C) {
#pragma omp parallel for schedule(static)
    for (int64_t row = 0; row < B; ++row) {
        const float *x = logits + row * C;
        float maxv = x[0];
        for (int64_t c = 1; c < C; ++c) if (x[c] > maxv) maxv = x[c];
        float s = 0.0f;
        for (int64_t c = 0; c < C; ++c) s = s + expf(x[c] - maxv);
        uint32_t t = or_ce_target(targets[row], C);
        float log_denom = maxv + logf(s);
        loss[row] = log_denom - x[t];
    }
}

/* cross_entropy_backward.wgsl:12-56 with reductionOps.ts:491-531 packing:
 * scale = 1/B for "mean", else 1; upstream = go[0] if go has one element.   */
OR_EXPORT void or_cross_entropy_backward(const float *go, int go_is_scalar, const float *logits,
                                         const float *targets, float *gi, int64_t B, int64_t C, float scale) {
#pragma omp parallel for schedule(static)
    for (int64_t idx = 0; idx < B * C; ++idx) {
        int64_t row = idx / C, col = idx % C;
        const float *x = logits + row * C;
        float maxv = x[0];
        for (int64_t c = 1; c < C; ++c) if (x[c] > maxv) maxv = x[c];
        float s = 0.0f;
        for (int64_t c = 0; c < C; ++c) s = s + expf(x[c] - maxv);
        float prob = expf(logits[idx] - maxv) / s;
        uint32_t t = or_ce_target(targets[row], C);
        float one_hot = ((uint32_t)col == t) ? 1.0f : 0.0f;
        float up = go_is_scalar ? go[0] : go[row];
        float row_scale = up * scale;
        gi[idx] = (prob - one_hot) * row_scale;
    }
}

/* ------------------------------------------------------------------------- */
/* conv.wgsl:25-60 conv2d (convOps.ts:17-62): one output per invocation,
 * loop kc, kh, kw; padding taps skipped; dilation ignored; + bias[oc].       */
typedef struct {
    int64_t N, Cin, Cout, H, W, OH, OW, KH, KW, SH, SW, PH, PW, groups;
} or_conv_params;

OR_EXPORT void or_conv2d(const float *in, const float *w, const float *bias, float *out, const or_conv_params *p) {
    int64_t total = p->N * p->Cout * p->OH * p->OW;
    int64_t icpg = p->Cin / p->groups, ocpg = p->Cout / p->groups;
#pragma omp parallel for schedule(static)
    for (int64_t idx = 0; idx < total; ++idx) {
        int64_t ow = idx % p->OW, oh = (idx / p->OW) % p->OH;
        int64_t oc = (idx / (p->OW * p->OH)) % p->Cout, b = idx / (p->Cout * p->OH * p->OW);
        int64_t g = oc / ocpg;
        float sum = 0.0f;
        for (int64_t kc = 0; kc < icpg; ++kc) {
            int64_t ic = g * icpg + kc;
            for (int64_t kh = 0; kh < p->KH; ++kh) {
                int64_t ih = oh * p->SH + kh - p->PH;
                for (int64_t kw = 0; kw < p->KW; ++kw) {
                    int64_t iw = ow * p->SW + kw - p->PW;
                    if (ih >= 0 && ih < p->H && iw >= 0 && iw < p->W)
                        sum += in[((b * p->Cin + ic) * p->H + ih) * p->W + iw] *
                               w[((oc * icpg + kc) * p->KH + kh) * p->KW + kw];
                }
            }
        }
        sum += bias ? bias[oc] : 0.0f;
        out[idx] = sum;
    }
}

/* conv_backward.wgsl:24-61 conv2d_input_backward (groups forced to 1 by
 * convOps.ts:82): per input element, loop kh, kw, then oc.                   */
OR_EXPORT void or_conv2d_input_backward(const float *go, const float *w, float *gi, const or_conv_params *p) {
    int64_t total = p->N * p->Cin * p->H * p->W;
#pragma omp parallel for schedule(static)
    for (int64_t idx = 0; idx < total; ++idx) {
        int64_t iw = idx % p->W, ih = (idx / p->W) % p->H;
        int64_t ic = (idx / (p->W * p->H)) % p->Cin, b = idx / (p->Cin * p->H * p->W);
        float sum = 0.0f;
        for (int64_t kh = 0; kh < p->KH; ++kh) {
            for (int64_t kw = 0; kw < p->KW; ++kw) {
                int64_t ohb = ih + p->PH - kh, owb = iw + p->PW - kw;
                if (ohb >= 0 && owb >= 0 && ohb % p->SH == 0 && owb % p->SW == 0) {
                    int64_t oh = ohb / p->SH, ow = owb / p->SW;
                    if (oh < p->OH && ow < p->OW)
                        for (int64_t oc = 0; oc < p->Cout; ++oc)
                            sum += go[((b * p->Cout + oc) * p->OH + oh) * p->OW + ow] *
                                   w[((oc * p->Cin + ic) * p->KH + kh) * p->KW + kw];
                }
            }
        }
        gi[idx] = sum;
    }
}

/* conv_backward.wgsl:66-101 conv2d_weight_backward: per weight, loop b, oh, ow. */
OR_EXPORT void or_conv2d_weight_backward(const float *go, const float *in, float *gw, const or_conv_params *p) {
    int64_t total = p->Cout * p->Cin * p->KH * p->KW;
#pragma omp parallel for schedule(dynamic, 1)
    for (int64_t idx = 0; idx < total; ++idx) {
        int64_t kw = idx % p->KW, kh = (idx / p->KW) % p->KH;
        int64_t ic = (idx / (p->KW * p->KH)) % p->Cin, oc = idx / (p->KW * p->KH * p->Cin);
        float sum = 0.0f;
        for (int64_t b = 0; b < p->N; ++b)
            for (int64_t oh = 0; oh < p->OH; ++oh)
                for (int64_t ow = 0; ow < p->OW; ++ow) {
                    int64_t ih = oh * p->SH + kh - p->PH, iw = ow * p->SW + kw - p->PW;
                    if (ih >= 0 && ih < p->H && iw >= 0 && iw < p->W)
                        sum += go[((b * p->Cout + oc) * p->OH + oh) * p->OW + ow] *
                               in[((b * p->Cin + ic) * p->H + ih) * p->W + iw];
                }
        gw[idx] = sum;
    }
}

/* conv_backward.wgsl:103-119 conv2d_bias_backward: per channel, loop b, oh, ow. */
OR_EXPORT void or_conv2d_bias_backward(const float *go, float *gb, int64_t N, int64_t C, int64_t OH, int64_t OW) {
#pragma omp parallel for schedule(static)
    for (int64_t c = 0; c < C; ++c) {
        float sum = 0.0f;
        for (int64_t b = 0; b < N; ++b)
            for (int64_t i = 0; i < OH * OW; ++i) sum += go[(b * C + c) * OH * OW + i];
        gb[c] = sum;
    }
}

/* ------------------------------------------------------------------------- */
/* max_pool2d.wgsl:22-49: init -3.402823e38, strict >, padded taps skipped.
 * idx (may be NULL) receives the flat ih*W+iw of the first maximum within the
 * (b,c) plane; the reference has no index output and no backward (it never
 * registers an autograd node, tensor_nn_ops.py:57-72).  The index is the
 * PyTorch convention, restated here as the intended semantics.               */
typedef struct {
    int64_t N, C, H, W, OH, OW, KH, KW, SH, SW, PH, PW, DH, DW;
} or_pool_params;

OR_EXPORT void or_max_pool2d(const float *in, float *out, int32_t *idx, const or_pool_params *p) {
    int64_t total = p->N * p->C * p->OH * p->OW;
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < total; ++i) {
        int64_t ow = i % p->OW, oh = (i / p->OW) % p->OH, bc = i / (p->OW * p->OH);
        float m = -3.402823e+38f;
        int32_t mi = -1;
        for (int64_t kh = 0; kh < p->KH; ++kh) {
            int64_t ih = oh * p->SH + kh * p->DH - p->PH;
            for (int64_t kw = 0; kw < p->KW; ++kw) {
                int64_t iw = ow * p->SW + kw * p->DW - p->PW;
                if (ih >= 0 && ih < p->H && iw >= 0 && iw < p->W) {
                    float v = in[(bc * p->H + ih) * p->W + iw];
                    if (v > m) { m = v; mi = (int32_t)(ih * p->W + iw); }
                }
            }
        }
        out[i] = m;
        if (idx) idx[i] = mi;
    }
}

/* Max-pool backward (new; the PyTorch rule): each output gradient goes to the
 * input position recorded in idx; overlapping windows accumulate in output
 * order.                                                                      */
OR_EXPORT void or_max_pool2d_backward(const float *go, const int32_t *idx, float *gi, const or_pool_params *p) {
    int64_t planes = p->N * p->C, in_plane = p->H * p->W, out_plane = p->OH * p->OW;
    memset(gi, 0, sizeof(float) * (size_t)(planes * in_plane));
#pragma omp parallel for schedule(static)
    for (int64_t bc = 0; bc < planes; ++bc)
        for (int64_t o = 0; o < out_plane; ++o) {
            int32_t j = idx[bc * out_plane + o];
            if (j >= 0) gi[bc * in_plane + j] += go[bc * out_plane + o];
        }
}

/* ------------------------------------------------------------------------- */
/* batchnorm.wgsl:20-36 (inference): (x-mean)*inv_std*w+b with
 * inv_std = 1/sqrt(var+eps); normalizationOps.ts:20-126 packs missing weight
 * as 1, bias/mean as 0, var as 1.                                            */
OR_EXPORT void or_batchnorm_eval(const float *x, const float *w, const float *b, const float *rm, const float *rv,
                                 float *y, int64_t N, int64_t C, int64_t S, float eps) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < N * C * S; ++i) {
        int64_t c = (i / S) % C;
        float wt = w ? w[c] : 1.0f, bs = b ? b[c] : 0.0f, mean = rm ? rm[c] : 0.0f, var = rv ? rv[c] : 1.0f;
        float inv_std = 1.0f / sqrtf(var + eps);
        y[i] = (x[i] - mean) * inv_std * wt + bs;
    }
}

/* BatchNorm training forward, the math of tensor_nn_ops.py:92-254 (batch mean
 * and biased variance over N and the spatial dims, x_hat=(x-mean)*rsqrt(var+
 * eps), affine, running stats updated with momentum and the unbiased variance
 * var*M/(M-1), :206-217).  Statistics accumulate in f64 here so the oracle is
 * an accurate anchor for a single-pass device Welford; saves mean and
 * inv_std per channel for the backward.                                      */
OR_EXPORT void or_batchnorm_train(const float *x, const float *w, const float *b, float *rm, float *rv, float *y,
                                  float *save_mean, float *save_invstd, int64_t N, int64_t C, int64_t S, float eps,
                                  float momentum) {
    double M = (double)(N * S);
#pragma omp parallel for schedule(static)
    for (int64_t c = 0; c < C; ++c) {
        double s = 0.0, ss = 0.0;
        for (int64_t n = 0; n < N; ++n)
            for (int64_t i = 0; i < S; ++i) s += x[(n * C + c) * S + i];
        double mean = s / M;
        for (int64_t n = 0; n < N; ++n)
            for (int64_t i = 0; i < S; ++i) { double d = x[(n * C + c) * S + i] - mean; ss += d * d; }
        double var = ss / M;
        float inv_std = (float)(1.0 / sqrt(var + (double)eps));
        float fm = (float)mean;
        float wt = w ? w[c] : 1.0f, bs = b ? b[c] : 0.0f;
        for (int64_t n = 0; n < N; ++n)
            for (int64_t i = 0; i < S; ++i) {
                int64_t k = (n * C + c) * S + i;
                y[k] = (x[k] - fm) * inv_std * wt + bs;
            }
        if (save_mean) save_mean[c] = fm;
        if (save_invstd) save_invstd[c] = inv_std;
        if (rm) rm[c] = (float)(mean * momentum + rm[c] * (1.0 - momentum));
        if (rv) rv[c] = (float)(var * M / (M - 1.0) * momentum + rv[c] * (1.0 - momentum));
    }
}

/* BatchNorm training backward (PyTorch rule; the reference's composite
 * autograd_rules.py:1049-1130 differs: it throws for W != C and scales the
 * parameter grads by gamma).  dx = w*inv_std*(dy - mean(dy) - x_hat*mean(dy*x_hat)),
 * dw = sum(dy*x_hat), db = sum(dy).  f64 accumulation.                        */
OR_EXPORT void or_batchnorm_backward(const float *dy, const float *x, const float *w, const float *save_mean,
                                     const float *save_invstd, float *dx, float *dw, float *db, int64_t N, int64_t C,
                                     int64_t S) {
    double M = (double)(N * S);
#pragma omp parallel for schedule(static)
    for (int64_t c = 0; c < C; ++c) {
        double sdy = 0.0, sdyx = 0.0;
        double mean = save_mean[c], is = save_invstd[c];
        for (int64_t n = 0; n < N; ++n)
            for (int64_t i = 0; i < S; ++i) {
                int64_t k = (n * C + c) * S + i;
                sdy += dy[k];
                sdyx += dy[k] * (x[k] - mean) * is;
            }
        double wt = w ? w[c] : 1.0;
        for (int64_t n = 0; n < N; ++n)
            for (int64_t i = 0; i < S; ++i) {
                int64_t k = (n * C + c) * S + i;
                double xh = (x[k] - mean) * is;
                dx[k] = (float)(wt * is * (dy[k] - sdy / M - xh * sdyx / M));
            }
        if (dw) dw[c] = (float)sdyx;
        if (db) db[c] = (float)sdy;
    }
}

/* layernorm.wgsl:14-42 (no-grad path): per row, mean, then biased variance
 * in a second pass, inv_std = 1/sqrt(var+eps), gamma*x_hat+beta.  Optional
 * mean/rstd outputs feed the backward.                                       */
OR_EXPORT void or_layernorm(const float *x, const float *g, const float *b, float *y, float *save_mean,
                            float *save_rstd, int64_t rows, int64_t D, float eps) {
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; ++r) {
        const float *xr = x + r * D;
        float sum = 0.0f;
        for (int64_t i = 0; i < D; ++i) sum += xr[i];
        float mean = sum / (float)D;
        float vs = 0.0f;
        for (int64_t i = 0; i < D; ++i) { float d = xr[i] - mean; vs += d * d; }
        float var = vs / (float)D;
        float inv_std = 1.0f / sqrtf(var + eps);
        for (int64_t i = 0; i < D; ++i) {
            float nrm = (xr[i] - mean) * inv_std;
            y[r * D + i] = (g ? g[i] : 1.0f) * nrm + (b ? b[i] : 0.0f);
        }
        if (save_mean) save_mean[r] = mean;
        if (save_rstd) save_rstd[r] = inv_std;
    }
}

/* LayerNorm backward (PyTorch rule; the reference composite
 * autograd_rules.py:1133-1209 scales dgamma/dbeta by gamma, D4):
 * dx = rstd*(g*dy - mean(g*dy) - x_hat*mean(g*dy*x_hat)), dgamma = sum_rows
 * dy*x_hat, dbeta = sum_rows dy.  f64 accumulation.                          */
OR_EXPORT void or_layernorm_backward(const float *dy, const float *x, const float *g, const float *save_mean,
                                     const float *save_rstd, float *dx, float *dg, float *db, int64_t rows, int64_t D) {
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; ++r) {
        double mean = save_mean[r], rs = save_rstd[r];
        double a = 0.0, bsum = 0.0;
        for (int64_t i = 0; i < D; ++i) {
            double xh = (x[r * D + i] - mean) * rs;
            double gd = (g ? g[i] : 1.0) * dy[r * D + i];
            a += gd;
            bsum += gd * xh;
        }
        for (int64_t i = 0; i < D; ++i) {
            double xh = (x[r * D + i] - mean) * rs;
            double gd = (g ? g[i] : 1.0) * dy[r * D + i];
            dx[r * D + i] = (float)(rs * (gd - a / D - xh * bsum / D));
        }
    }
    if (dg || db) {
#pragma omp parallel for schedule(static)
        for (int64_t i = 0; i < D; ++i) {
            double sg = 0.0, sb = 0.0;
            for (int64_t r = 0; r < rows; ++r) {
                double xh = (x[r * D + i] - save_mean[r]) * save_rstd[r];
                sg += dy[r * D + i] * xh;
                sb += dy[r * D + i];
            }
            if (dg) dg[i] = (float)sg;
            if (db) db[i] = (float)sb;
        }
    }
}

/* ------------------------------------------------------------------------- */
/* adamw_step.wgsl:11-40 (reductionOps.ts:579-623).  All hyper-parameters
 * arrive as f32 uniforms; step_size and inv_sqrt_bc2 were computed on the
 * host in f64 (optim/__init__.py:385-388) and rounded to f32.                */
OR_EXPORT void or_adamw_step(float *param, const float *grad, float *m_, float *v_, int64_t n, float lr, float beta1,
                             float beta2, float eps, float wd, float step_size, float inv_sqrt_bc2) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) {
        float p = param[i];
        if (wd != 0.0f) p = p - (lr * wd) * p;
        float g = grad[i];
        float m = m_[i] * beta1 + (1.0f - beta1) * g;
        float v = v_[i] * beta2 + (1.0f - beta2) * g * g;
        m_[i] = m;
        v_[i] = v;
        float denom = sqrtf(v) * inv_sqrt_bc2 + eps;
        float update = (m / denom) * step_size;
        param[i] = p - update;
    }
}

/* adam_step.wgsl:11-39: L2 weight decay folded into the gradient.           */
OR_EXPORT void or_adam_step(float *param, const float *grad, float *m_, float *v_, int64_t n, float lr, float beta1,
                            float beta2, float eps, float wd, float step_size, float inv_sqrt_bc2) {
    (void)lr;
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) {
        float p = param[i];
        float g = grad[i];
        if (wd != 0.0f) g = g + wd * p;
        float m = m_[i] * beta1 + (1.0f - beta1) * g;
        float v = v_[i] * beta2 + (1.0f - beta2) * g * g;
        m_[i] = m;
        v_[i] = v;
        float denom = sqrtf(v) * inv_sqrt_bc2 + eps;
        float update = (m / denom) * step_size;
        param[i] = p - update;
    }
}

/* sgd_step.wgsl:9-42 (reductionOps.ts:625-653): has_momentum = momentum != 0;
 * the momentum buffer starts at zeros (optim/__init__.py:177-179).           */
OR_EXPORT void or_sgd_step(float *param, const float *grad, float *buf_, int64_t n, float lr, float momentum, float wd,
                           float dampening, int nesterov) {
    int has_m = momentum != 0.0f;
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) {
        float g = grad[i];
        float p = param[i];
        if (wd != 0.0f) g = g + wd * p;
        float update = g;
        if (has_m) {
            float buf = buf_[i];
            buf = buf * momentum + g * (1.0f - dampening);
            buf_[i] = buf;
            update = nesterov ? g + momentum * buf : buf;
        }
        param[i] = p - lr * update;
    }
}

/* ------------------------------------------------------------------------- */
/* rmsprop_step.wgsl:11-42 (reductionOps.ts:655-688): use_momentum is
 * momentum != 0; the momentum buffer is read and written only then.         */
OR_EXPORT void or_rmsprop_step(float *param, const float *grad, float *sq_, float *mb_, int64_t n, float lr,
                               float alpha, float eps, float wd, float momentum) {
    int use_m = momentum != 0.0f;
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) {
        float p = param[i];
        float g = grad[i];
        if (wd != 0.0f) g = g + wd * p;
        float sq = sq_[i] * alpha + (1.0f - alpha) * g * g;
        sq_[i] = sq;
        float denom = sqrtf(sq) + eps;
        float update = g / denom;
        if (use_m) {
            float buf = mb_[i] * momentum + update;
            mb_[i] = buf;
            update = buf;
        }
        param[i] = p - lr * update;
    }
}

/* extended_step.wgsl adagrad_step (reductionOps.ts:690-737): hp = [lr, 0, 0,
 * eps], extra = [weight_decay, ...].                                         */
OR_EXPORT void or_adagrad_step(float *param, const float *grad, float *sum_, int64_t n, float lr, float eps,
                               float wd) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) {
        float p = param[i];
        float g = grad[i];
        if (wd != 0.0f) g = g + wd * p;
        float s = sum_[i] + g * g;
        sum_[i] = s;
        float sd = sqrtf(s) + eps;
        param[i] = p - lr * g / sd;
    }
}

/* extended_step.wgsl adamax_step (reductionOps.ts:739-780): extra =
 * [weight_decay, step_size, bias_correction1, 0].                           */
OR_EXPORT void or_adamax_step(float *param, const float *grad, float *m_, float *u_, int64_t n, float lr, float beta1,
                              float beta2, float eps, float wd, float step_size, float bc1) {
    (void)lr;
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) {
        float p = param[i];
        float g = grad[i];
        if (wd != 0.0f) g = g + wd * p;
        float m = m_[i] * beta1 + (1.0f - beta1) * g;
        float u = fmaxf(u_[i] * beta2, fabsf(g));
        m_[i] = m;
        u_[i] = u;
        float denom = u + eps;
        float update = (m / denom) * step_size * bc1;
        param[i] = p - update;
    }
}

/* extended_step.wgsl nadam_step (reductionOps.ts:782-823): extra =
 * [weight_decay, step_size, mu, 0]; m_hat = mu m + (1 - mu) g.               */
OR_EXPORT void or_nadam_step(float *param, const float *grad, float *m_, float *v_, int64_t n, float lr, float beta1,
                             float beta2, float eps, float wd, float step_size, float mu) {
    (void)lr;
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) {
        float p = param[i];
        float g = grad[i];
        if (wd != 0.0f) g = g + wd * p;
        float m = m_[i] * beta1 + (1.0f - beta1) * g;
        float v = v_[i] * beta2 + (1.0f - beta2) * g * g;
        m_[i] = m;
        v_[i] = v;
        float m_hat = mu * m + (1.0f - mu) * g;
        float denom = sqrtf(v) + eps;
        float update = (m_hat / denom) * step_size;
        param[i] = p - update;
    }
}

/* extended_step.wgsl radam_step (reductionOps.ts:825-868): extra =
 * [weight_decay, step_size, beta1^t, beta2^t], t = max(f32(step), 1).        */
OR_EXPORT void or_radam_step(float *param, const float *grad, float *m_, float *v_, int64_t n, float lr, float beta1,
                             float beta2, float eps, float wd, float step_size, float b1pow, float b2pow,
                             int64_t step) {
    (void)lr;
    (void)eps;
    float t_int = (float)(uint32_t)step;
    if (t_int < 1.0f) t_int = 1.0f;
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) {
        float p = param[i];
        float g = grad[i];
        if (wd != 0.0f) g = g + wd * p;
        float m = m_[i] * beta1 + (1.0f - beta1) * g;
        float v = v_[i] * beta2 + (1.0f - beta2) * g * g;
        m_[i] = m;
        v_[i] = v;
        float m_hat = m / (1.0f - b1pow);
        float rho_inf = 2.0f / (1.0f - beta2) - 1.0f;
        float one_minus_b2t = 1.0f - b2pow;
        float rho_t = rho_inf - 2.0f * t_int * b2pow / fmaxf(one_minus_b2t, 1e-10f);
        float update;
        if (rho_t > 5.0f) {
            float rect = sqrtf((rho_t - 4.0f) * (rho_t - 2.0f) * rho_inf / ((rho_inf - 4.0f) * (rho_inf - 2.0f) * rho_t));
            update = step_size * m_hat * rect;
        } else {
            update = step_size * m_hat;
        }
        param[i] = p - update;
    }
}
