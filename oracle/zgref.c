/*
 * zgref.c -- CPU oracle (test infrastructure only; see zgref.h).
 *
 * Reference call sites restated here:
 *   step_key      src/zerograd/_keys.py:20-30   (crc32 of "seed:run:version:generation")
 *   candidate_key src/zerograd/_keys.py:33-53   (jax.random.fold_in)
 *   group_key     src/zerograd/_keys.py:56-58   (jax.random.split(ck, n)[g])
 *   matrix/table/vector factors src/zerograd/_factors.py:43-74
 * and the published algorithms of the third-party code those lines call.
 */
#include "zgref.h"
#include <math.h>
#include <string.h>
#include <pthread.h>
#include <unistd.h>
#include <stdlib.h>

/* ---- a small pthread parallel-for (libgomp is not available here) ----- */
static int g_threads = 0;

int zgo_num_threads(void) {
    if (g_threads <= 0) {
        const char* e = getenv("ZGO_THREADS");
        long n = e ? strtol(e, NULL, 10) : sysconf(_SC_NPROCESSORS_ONLN);
        g_threads = n < 1 ? 1 : (n > 256 ? 256 : (int)n);
    }
    return g_threads;
}

void zgo_set_num_threads(int n) { g_threads = n < 1 ? 1 : n; }

typedef void (*range_fn)(void* ctx, int64_t begin, int64_t end);
typedef struct { range_fn fn; void* ctx; int64_t begin, end; } range_job;

static void* run_range(void* p) {
    range_job* j = (range_job*)p;
    j->fn(j->ctx, j->begin, j->end);
    return NULL;
}

static void parallel_for(int64_t n, int64_t min_per_thread, range_fn fn, void* ctx) {
    int t = zgo_num_threads();
    if (min_per_thread < 1) min_per_thread = 1;
    if ((int64_t)t > n / min_per_thread) t = (int)(n / min_per_thread);
    if (t <= 1) { fn(ctx, 0, n); return; }
    pthread_t th[256];
    range_job jobs[256];
    int64_t chunk = (n + t - 1) / t;
    for (int i = 0; i < t; ++i) {
        int64_t b = i * chunk, e = b + chunk < n ? b + chunk : n;
        jobs[i] = (range_job){fn, ctx, b, e};
        if (b >= e) continue;
        if (i == 0) continue;
        if (pthread_create(&th[i], NULL, run_range, &jobs[i]) != 0) {
            fn(ctx, b, e); /* could not start a thread: run inline */
            jobs[i].begin = jobs[i].end;
        }
    }
    if (jobs[0].begin < jobs[0].end) fn(ctx, jobs[0].begin, jobs[0].end);
    for (int i = 1; i < t; ++i)
        if (jobs[i].begin < jobs[i].end) pthread_join(th[i], NULL);
}

/* ---- CRC-32 (ISO-HDLC / zlib polynomial 0xEDB88320, reflected) ------- */
uint32_t zgo_crc32(const uint8_t* data, size_t n) {
    uint32_t c = 0xFFFFFFFFu;
    for (size_t i = 0; i < n; ++i) {
        c ^= data[i];
        for (int b = 0; b < 8; ++b) c = (c >> 1) ^ (0xEDB88320u & (0u - (c & 1u)));
    }
    return c ^ 0xFFFFFFFFu;
}

/* ---- threefry2x32, 20 rounds ------------------------------------------ */
static inline uint32_t rotl32(uint32_t x, int r) { return (x << r) | (x >> (32 - r)); }

void zgo_threefry2x32(uint32_t k0, uint32_t k1, uint32_t c0, uint32_t c1, uint32_t out[2]) {
    static const int R[8] = {13, 15, 26, 6, 17, 29, 16, 24};
    const uint32_t ks[3] = {k0, k1, k0 ^ k1 ^ 0x1BD11BDAu};
    uint32_t x0 = c0 + ks[0], x1 = c1 + ks[1];
    for (int g = 0; g < 5; ++g) {
        const int* rot = R + 4 * (g & 1);
        for (int i = 0; i < 4; ++i) {
            x0 += x1;
            x1 = rotl32(x1, rot[i]);
            x1 ^= x0;
        }
        x0 += ks[(g + 1) % 3];
        x1 += ks[(g + 2) % 3] + (uint32_t)(g + 1);
    }
    out[0] = x0;
    out[1] = x1;
}

void zgo_fold_in(const uint32_t key[2], uint32_t d, uint32_t out[2]) {
    zgo_threefry2x32(key[0], key[1], 0u, d, out);
}

void zgo_split(const uint32_t key[2], int64_t n, uint32_t* out) {
    for (int64_t i = 0; i < n; ++i)
        zgo_threefry2x32(key[0], key[1], (uint32_t)((uint64_t)i >> 32), (uint32_t)i, out + 2 * i);
}

typedef struct { uint32_t k0, k1; uint32_t* out; } bits_ctx;

static void bits_range(void* c, int64_t b, int64_t e) {
    bits_ctx* x = (bits_ctx*)c;
    for (int64_t j = b; j < e; ++j) {
        uint32_t o[2];
        zgo_threefry2x32(x->k0, x->k1, (uint32_t)((uint64_t)j >> 32), (uint32_t)j, o);
        x->out[j] = o[0] ^ o[1];
    }
}

void zgo_random_bits32(const uint32_t key[2], int64_t n, uint32_t* out) {
    bits_ctx c = {key[0], key[1], out};
    parallel_for(n, 65536, bits_range, &c);
}

/* ---- uniform / normal --------------------------------------------------- */
static inline float f32_from_bits(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

float zgo_bits_to_uniform(uint32_t bits, float lo, float hi) {
    /* 23 random mantissa bits with exponent 0 -> [1,2), minus 1 -> [0,1) */
    float f = f32_from_bits((bits >> 9) | 0x3F800000u) - 1.0f;
    float span = hi - lo; /* float32 subtraction, as the traced computation does */
    float v = f * span + lo;
    return v > lo ? v : lo;
}

/* Giles, "Approximating the erfinv function" (GPU Computing Gems, 2011),
 * single-precision branch polynomials; Horner steps as explicit fmaf. */
float zgo_erfinv_f32(float x) {
    if (fabsf(x) == 1.0f) return x * INFINITY;
    float w = -log1pf(-x * x);
    float p;
    if (w < 5.0f) {
        w = w - 2.5f;
        p = 2.81022636e-08f;
        p = fmaf(p, w, 3.43273939e-07f);
        p = fmaf(p, w, -3.5233877e-06f);
        p = fmaf(p, w, -4.39150654e-06f);
        p = fmaf(p, w, 0.00021858087f);
        p = fmaf(p, w, -0.00125372503f);
        p = fmaf(p, w, -0.00417768164f);
        p = fmaf(p, w, 0.246640727f);
        p = fmaf(p, w, 1.50140941f);
    } else {
        w = sqrtf(w) - 3.0f;
        p = -0.000200214257f;
        p = fmaf(p, w, 0.000100950558f);
        p = fmaf(p, w, 0.00134934322f);
        p = fmaf(p, w, -0.00367342844f);
        p = fmaf(p, w, 0.00573950773f);
        p = fmaf(p, w, -0.0076224613f);
        p = fmaf(p, w, 0.00943887047f);
        p = fmaf(p, w, 1.00167406f);
        p = fmaf(p, w, 2.83297682f);
    }
    return p * x;
}

float zgo_bits_to_normal(uint32_t bits) {
    /* lo = nextafter(-1, 0) in float32 */
    const float lo = f32_from_bits(0xBF7FFFFFu);
    float u = zgo_bits_to_uniform(bits, lo, 1.0f);
    return 1.41421356237309504880f * zgo_erfinv_f32(u);
}

typedef struct { uint32_t k0, k1; float* out; } normal_ctx;

static void normal_range(void* c, int64_t b, int64_t e) {
    normal_ctx* x = (normal_ctx*)c;
    for (int64_t j = b; j < e; ++j) {
        uint32_t o[2];
        zgo_threefry2x32(x->k0, x->k1, (uint32_t)((uint64_t)j >> 32), (uint32_t)j, o);
        x->out[j] = zgo_bits_to_normal(o[0] ^ o[1]);
    }
}

static void normal_serial(const uint32_t key[2], int64_t n, float* out) {
    normal_ctx c = {key[0], key[1], out};
    normal_range(&c, 0, n);
}

void zgo_normal_f32(const uint32_t key[2], int64_t n, float* out) {
    normal_ctx c = {key[0], key[1], out};
    parallel_for(n, 65536, normal_range, &c);
}

/* ---- factors ------------------------------------------------------------ */
static void split2(const uint32_t key[2], uint32_t ka[2], uint32_t kb[2]) {
    zgo_threefry2x32(key[0], key[1], 0u, 0u, ka);
    zgo_threefry2x32(key[0], key[1], 0u, 1u, kb);
}

void zgo_matrix_factors(const uint32_t gk[2], int64_t rows, int64_t cols, int rank,
                        float* A, float* B) {
    uint32_t ka[2], kb[2];
    split2(gk, ka, kb);
    zgo_normal_f32(ka, rows * (int64_t)rank, A); /* A[i,j] = normal(ka)[i*rank+j] */
    zgo_normal_f32(kb, (int64_t)rank * cols, B); /* B[j,o] = normal(kb)[j*cols+o] */
}

void zgo_table_factors(const uint32_t gk[2], int64_t rows, int64_t cols, int rank,
                       float* A, float* B) {
    uint32_t ka[2], kb[2];
    split2(gk, ka, kb);
    zgo_normal_f32(ka, rows * (int64_t)rank, A); /* A[x,j] */
    zgo_normal_f32(kb, cols * (int64_t)rank, B); /* B[y,j] */
}

void zgo_vector_noise(const uint32_t gk[2], int64_t n, float* out) { zgo_normal_f32(gk, n, out); }

void zgo_candidate_keys(const uint32_t base[2], const int32_t* ids, int64_t n, uint32_t* out) {
    for (int64_t i = 0; i < n; ++i) zgo_fold_in(base, (uint32_t)ids[i], out + 2 * i);
}

void zgo_group_keys(const uint32_t* cand_keys, int64_t n, int group, uint32_t* out) {
    for (int64_t i = 0; i < n; ++i) zgo_fold_in(cand_keys + 2 * i, (uint32_t)group, out + 2 * i);
}

typedef struct {
    const uint32_t* gks; int layout; int64_t rows, cols; int rank; float *A, *B;
} pop_ctx;

static void pop_range(void* c, int64_t b, int64_t e) {
    pop_ctx* x = (pop_ctx*)c;
    for (int64_t p = b; p < e; ++p) {
        const uint32_t* gk = x->gks + 2 * p;
        if (x->layout == 2) {
            normal_serial(gk, x->rows, x->A + p * x->rows);
            continue;
        }
        uint32_t ka[2], kb[2];
        split2(gk, ka, kb);
        int64_t na = x->rows * x->rank, nb = x->cols * x->rank;
        normal_serial(ka, na, x->A + p * na);
        normal_serial(kb, nb, x->B + p * nb); /* [rank,cols] (matrix) or [cols,rank] (table): same flat count */
    }
}

void zgo_population_factors(const uint32_t* gks, int64_t P, int layout,
                            int64_t rows, int64_t cols, int rank, float* A, float* B) {
    pop_ctx c = {gks, layout, rows, cols, rank, A, B};
    parallel_for(P, 1, pop_range, &c);
}

float zgo_round_bf16(float x) {
    uint32_t u;
    memcpy(&u, &x, 4);
    if ((u & 0x7F800000u) == 0x7F800000u) { /* inf / nan */
        if (u & 0x007FFFFFu) u |= 0x00400000u;
        u &= 0xFFFF0000u;
    } else {
        u += 0x7FFFu + ((u >> 16) & 1u);
        u &= 0xFFFF0000u;
    }
    return f32_from_bits(u);
}

/* ---- int8 GEMM + LUT ---------------------------------------------------- */
typedef struct {
    const int8_t *x, *W; const float* w_scale; float x_scale, y_scale; const int8_t* lut;
    const float *A, *Bf; int rank; float s; int64_t M, K, N; int8_t* out; int32_t* acc_out;
} i8_ctx;

static void i8_range(void* c, int64_t b, int64_t e) {
    const i8_ctx* a = (const i8_ctx*)c;
    const int64_t K = a->K, N = a->N;
    for (int64_t m = b; m < e; ++m) {
        float u[64];
        for (int j = 0; j < a->rank; ++j) {
            float t = 0.0f;
            for (int64_t k = 0; k < K; ++k) t = fmaf((float)a->x[m * K + k], a->A[k * a->rank + j], t);
            u[j] = t;
        }
        for (int64_t n = 0; n < N; ++n) {
            int64_t acc = 0;
            for (int64_t k = 0; k < K; ++k) acc += (int64_t)a->x[m * K + k] * (int64_t)a->W[k * N + n];
            if (a->acc_out) a->acc_out[m * N + n] = (int32_t)acc;
            float lr = 0.0f;
            for (int j = 0; j < a->rank; ++j) lr = fmaf(u[j], a->Bf[j * N + n], lr);
            float y = fmaf((float)acc * a->x_scale, a->w_scale[n], a->s * lr);
            float qf = rintf(y / a->y_scale);
            /* a NaN pre-activation quantises to 0 (defined here; the C cast is not) */
            int q = qf != qf ? 0 : (qf > 127.0f ? 127 : (qf < -128.0f ? -128 : (int)qf));
            a->out[m * N + n] = a->lut[q + 128];
        }
    }
}

void zgo_int8_lut_linear(const int8_t* x, const int8_t* W, const float* w_scale,
                         float x_scale, float y_scale, const int8_t* lut,
                         const float* A, const float* Bf, int rank, float s,
                         int64_t M, int64_t K, int64_t N, int8_t* out, int32_t* acc_out) {
    i8_ctx c = {x, W, w_scale, x_scale, y_scale, lut, A, Bf, rank, s, M, K, N, out, acc_out};
    parallel_for(M, 1, i8_range, &c);
}
