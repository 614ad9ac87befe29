/*
 * CPU restatement of the reference Gated DeltaNet recurrence in plain C.
 *
 * TEST INFRASTRUCTURE ONLY: this is the checker and the timed CPU baseline
 * ("port" of the reference's algorithm), never part of the shipped CUDA path.
 *
 * Follows the reference Triton kernels operation by operation:
 *   gates          solution/triton/kernel_decode.py:46-55, kernel_prefill.py:108-113
 *   decode step    solution/triton/kernel_decode.py:71-103
 *   prefill loop   solution/triton/kernel_prefill.py:55-142 (empty sequence:
 *                  initial state passes through, kernel_prefill.py:65-73)
 *   default scale  kernel_decode.py:124-125 (scale <= 0 -> 1/sqrt(d))
 *   zero state     kernel_decode.py:133-143 (state == NULL)
 *   GVA mapping    qk_head = v_head / (HV / HQ)   (kernel_decode.py:44 with ratio 2)
 *
 * Work is split over (sequence, v-head) units with POSIX threads; every unit is
 * independent, so the result does not depend on the thread count.
 * bf16 values travel as uint16 bit patterns (round-to-nearest-even on output).
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

static inline float bf16_to_f32(uint16_t h) {
    uint32_t u = ((uint32_t)h) << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

static inline uint16_t f32_to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

/* kernel_decode.py:52-55 */
static inline void gate_values(float A_log, float a, float dt_bias, float b, float* g, float* beta) {
    float x = a + dt_bias;
    float sp = x > 20.0f ? x : logf(1.0f + expf(x));
    *g = expf(-expf(A_log) * sp);
    *beta = 1.0f / (1.0f + expf(-b));
}

static void load_vec(const uint16_t* src, int D, int l2norm, float* dst) {
    float ss = 0.0f;
    for (int i = 0; i < D; ++i) {
        dst[i] = bf16_to_f32(src[i]);
        ss += dst[i] * dst[i];
    }
    if (l2norm) {
        float r = 1.0f / sqrtf(ss + 1e-6f);
        for (int i = 0; i < D; ++i) dst[i] *= r;
    }
}

/* One recurrence step over the D x D k-last state S (rows = v index),
 * kernel_decode.py:83-87. */
static void step(float* S, const float* k, const float* q, const uint16_t* v, float g, float beta,
                 float scale, int D, uint16_t* out) {
    for (int r = 0; r < D; ++r) {
        float* row = S + (size_t)r * D;
        float old_v = 0.0f;
        for (int c = 0; c < D; ++c) {
            row[c] *= g;
            old_v += row[c] * k[c];
        }
        float delta = beta * (bf16_to_f32(v[r]) - old_v);
        float o = 0.0f;
        for (int c = 0; c < D; ++c) {
            row[c] += delta * k[c];
            o += row[c] * q[c];
        }
        out[r] = f32_to_bf16(scale * o);
    }
}

typedef struct {
    /* shared problem description */
    const uint16_t *q, *k, *v, *a, *b;
    const float *state, *A_log, *dt_bias;
    const int64_t* cu; /* NULL for decode (one token per sequence) */
    uint16_t* out;
    float* new_state;
    int N, HQ, HV, D, l2norm;
    float scale;
    /* work split */
    int next_unit;
    pthread_mutex_t lock;
} Problem;

static void run_unit(Problem* p, int unit, float* kbuf, float* qbuf) {
    int n = unit / p->HV, h = unit % p->HV;
    int D = p->D, HV = p->HV, HQ = p->HQ;
    int qh = h / (HV / HQ);
    size_t sd = (size_t)D * D;
    float* S = p->new_state + ((size_t)n * HV + h) * sd;
    if (p->state)
        memcpy(S, p->state + ((size_t)n * HV + h) * sd, sd * sizeof(float));
    else
        memset(S, 0, sd * sizeof(float));
    int64_t t0 = p->cu ? p->cu[n] : n, t1 = p->cu ? p->cu[n + 1] : n + 1;
    for (int64_t t = t0; t < t1; ++t) {
        load_vec(p->k + ((size_t)t * HQ + qh) * D, D, p->l2norm, kbuf);
        load_vec(p->q + ((size_t)t * HQ + qh) * D, D, p->l2norm, qbuf);
        float g, beta;
        gate_values(p->A_log[h], bf16_to_f32(p->a[(size_t)t * HV + h]), p->dt_bias[h],
                    bf16_to_f32(p->b[(size_t)t * HV + h]), &g, &beta);
        step(S, kbuf, qbuf, p->v + ((size_t)t * HV + h) * D, g, beta, p->scale, D,
             p->out + ((size_t)t * HV + h) * D);
    }
}

static void* worker(void* arg) {
    Problem* p = (Problem*)arg;
    float* buf = (float*)malloc(sizeof(float) * 2 * (size_t)p->D);
    for (;;) {
        pthread_mutex_lock(&p->lock);
        int unit = p->next_unit++;
        pthread_mutex_unlock(&p->lock);
        if (unit >= p->N * p->HV) break;
        run_unit(p, unit, buf, buf + p->D);
    }
    free(buf);
    return NULL;
}

static int run_problem(Problem* p, int nthreads) {
    if (p->HQ <= 0 || p->HV % p->HQ != 0 || p->D <= 0) return 1;
    if (!(p->scale > 0.0f)) p->scale = 1.0f / sqrtf((float)p->D);
    p->next_unit = 0;
    pthread_mutex_init(&p->lock, NULL);
    if (nthreads < 1) nthreads = 1;
    pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * (size_t)nthreads);
    for (int i = 0; i < nthreads; ++i) pthread_create(&th[i], NULL, worker, p);
    for (int i = 0; i < nthreads; ++i) pthread_join(th[i], NULL);
    free(th);
    pthread_mutex_destroy(&p->lock);
    return 0;
}

/* Decode: q,k [B,HQ,D]; v [B,HV,D]; a,b [B,HV]; state [B,HV,D,D] or NULL. */
int gdn_oracle_decode(const uint16_t* q, const uint16_t* k, const uint16_t* v, const float* state,
                      const float* A_log, const uint16_t* a, const float* dt_bias, const uint16_t* b,
                      float scale, int use_qk_l2norm, uint16_t* out, float* new_state, int B, int HQ,
                      int HV, int D, int nthreads) {
    Problem p = {.q = q, .k = k, .v = v, .a = a, .b = b, .state = state, .A_log = A_log,
                 .dt_bias = dt_bias, .cu = NULL, .out = out, .new_state = new_state, .N = B,
                 .HQ = HQ, .HV = HV, .D = D, .l2norm = use_qk_l2norm, .scale = scale};
    return run_problem(&p, nthreads);
}

/* Prefill: q,k [T,HQ,D]; v [T,HV,D]; a,b [T,HV]; state [N,HV,D,D] or NULL; cu [N+1]. */
int gdn_oracle_prefill(const uint16_t* q, const uint16_t* k, const uint16_t* v, const float* state,
                       const float* A_log, const uint16_t* a, const float* dt_bias, const uint16_t* b,
                       const int64_t* cu_seqlens, float scale, int use_qk_l2norm, uint16_t* out,
                       float* new_state, int N, int HQ, int HV, int D, int nthreads) {
    for (int n = 0; n < N; ++n)
        if (cu_seqlens[n + 1] < cu_seqlens[n]) return 1;
    Problem p = {.q = q, .k = k, .v = v, .a = a, .b = b, .state = state, .A_log = A_log,
                 .dt_bias = dt_bias, .cu = cu_seqlens, .out = out, .new_state = new_state, .N = N,
                 .HQ = HQ, .HV = HV, .D = D, .l2norm = use_qk_l2norm, .scale = scale};
    return run_problem(&p, nthreads);
}
