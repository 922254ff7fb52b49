/*
 * synth.c — seeded synthetic tensors for the benchmark workloads.
 *
 * Counter-based: element i of a stream depends only on (seed, i), so any
 * thread split gives the same bytes. A normal sample is Box-Muller on two
 * splitmix64 hashes evaluated in double precision on the host.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <string.h>
#include <unistd.h>

static inline uint64_t splitmix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

static inline double normal_at(uint64_t seed, uint64_t i) {
    uint64_t k = splitmix64(seed * 0xD1B54A32D192ED03ull + 0x8CB92BA72F3D8DD7ull);
    uint64_t a = splitmix64(k ^ (2 * i));
    uint64_t b = splitmix64(k ^ (2 * i + 1));
    double u1 = ((double)(a >> 11) + 0.5) * (1.0 / 9007199254740992.0);
    double u2 = ((double)(b >> 11) + 0.5) * (1.0 / 9007199254740992.0);
    return sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2);
}

static inline uint16_t f32_to_bf16_rne(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

typedef struct {
    void *out;
    size_t lo, hi;
    uint64_t seed;
    float mean, std;
    int kind; /* 0 bf16, 1 f32, 2 f32 bf16-exact */
} job_t;

static void *run(void *p) {
    job_t *j = (job_t *)p;
    for (size_t i = j->lo; i < j->hi; i++) {
        float v = (float)(j->mean + j->std * normal_at(j->seed, i));
        if (j->kind == 0) {
            ((uint16_t *)j->out)[i] = f32_to_bf16_rne(v);
        } else if (j->kind == 1) {
            ((float *)j->out)[i] = v;
        } else {
            uint32_t u = (uint32_t)f32_to_bf16_rne(v) << 16;
            memcpy((float *)j->out + i, &u, 4);
        }
    }
    return NULL;
}

static void fill(void *out, size_t n, uint64_t seed, float mean, float std, int kind) {
    long nc = sysconf(_SC_NPROCESSORS_ONLN);
    int nt = (int)(nc < 1 ? 1 : (nc > 32 ? 32 : nc));
    if (n < (1u << 16)) nt = 1;
    pthread_t th[32];
    job_t jobs[32];
    size_t per = (n + nt - 1) / nt;
    for (int t = 0; t < nt; t++) {
        size_t lo = per * t, hi = lo + per;
        if (lo > n) lo = n;
        if (hi > n) hi = n;
        jobs[t] = (job_t){out, lo, hi, seed, mean, std, kind};
        if (nt == 1) run(&jobs[t]);
        else pthread_create(&th[t], NULL, run, &jobs[t]);
    }
    if (nt > 1)
        for (int t = 0; t < nt; t++) pthread_join(th[t], NULL);
}

void ds_synth_normal_bf16(uint16_t *out, size_t n, uint64_t seed, float mean, float stddev) {
    fill(out, n, seed, mean, stddev, 0);
}
void ds_synth_normal_f32(float *out, size_t n, uint64_t seed, float mean, float stddev) {
    fill(out, n, seed, mean, stddev, 1);
}
void ds_synth_normal_f32_bf16exact(float *out, size_t n, uint64_t seed, float mean, float stddev) {
    fill(out, n, seed, mean, stddev, 2);
}
