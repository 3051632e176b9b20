/*
 * sampling.c -- CPU restatement of the reference's temperature sampling.
 *
 * TEST INFRASTRUCTURE ONLY (see oracle.h).
 *
 * The reference (src/main.cpp:91-111, static sample_temperature) does, per
 * token:
 *   temperature <= 0      -> sample_argmax (main.cpp:79-89);
 *   max = logits[0], then strict '>' over the rest (main.cpp:94-96);
 *   probs[i] = exp((double)((logits[i] - max) / temperature)), the
 *              subtraction and division in float, exp in double (:98-102);
 *   sum = probs[0] + probs[1] + ... in double, in order (:100-103);
 *   probs[i] /= sum (:105);
 *   std::discrete_distribution<int> dist(probs) and dist(rng) with a
 *   std::mt19937 seeded from std::random_device (:107-110).
 * The distribution and the generator live in libstdc++ (GCC 13's <random>,
 * bits/random.tcc: discrete_distribution::param_type::_M_initialize,
 * discrete_distribution::operator(), generate_canonical), restated here:
 *   - fewer than two weights: no table, the draw is 0 without using the
 *     generator;
 *   - __sum = accumulate(probs, 0.0) (in order), every weight divided by
 *     __sum, cp = partial_sum (in order), cp[n - 1] = 1.0;
 *   - u = generate_canonical<double, 53>(mt19937): two 32-bit outputs g1, g2,
 *     sum = g1 + g2 * 2^32 (in double), u = sum / 2^64, and u >= 1 becomes
 *     nextafter(1, 0);
 *   - the draw is lower_bound(cp, u): the libstdc++ halving loop (first
 *     element not less than u), followed literally so that NaN tables give
 *     the library's answer.
 * mt19937 is the published MT19937 (Matsumoto and Nishimura, 1998) with the
 * standard's seeding (init_genrand).  The draws are deterministic given u,
 * which the device sampler takes as an input; tests/test_oracle.py pins this
 * restatement to the real libstdc++ (oracle/pin_sampling.cpp).
 */
#include "oracle.h"

#include <math.h>

#define ORC_OK 0
#define ORC_ERR_INVALID_ARG 8

/* ---- MT19937 ------------------------------------------------------------ */
void orc_mt_seed(orc_mt* st, uint32_t seed) {
    st->s[0] = seed;
    for (int i = 1; i < 624; i++)
        st->s[i] = 1812433253u * (st->s[i - 1] ^ (st->s[i - 1] >> 30)) + (uint32_t)i;
    st->i = 624;
}

uint32_t orc_mt_next(orc_mt* st) {
    if (st->i >= 624) {
        for (int k = 0; k < 624; k++) {
            const uint32_t y = (st->s[k] & 0x80000000u) | (st->s[(k + 1) % 624] & 0x7fffffffu);
            st->s[k] = st->s[(k + 397) % 624] ^ (y >> 1) ^ ((y & 1u) ? 0x9908b0dfu : 0u);
        }
        st->i = 0;
    }
    uint32_t y = st->s[st->i++];
    y ^= y >> 11;
    y ^= (y << 7) & 0x9d2c5680u;
    y ^= (y << 15) & 0xefc60000u;
    y ^= y >> 18;
    return y;
}

/* generate_canonical<double, 53> over a 32-bit generator: two outputs. */
double orc_canonical53(orc_mt* st) {
    double sum = 0.0, tmp = 1.0;
    for (int k = 2; k != 0; --k) {
        sum += (double)orc_mt_next(st) * tmp;
        tmp *= 4294967296.0;
    }
    double ret = sum / tmp;
    if (ret >= 1.0) ret = nextafter(1.0, 0.0);
    return ret;
}

void orc_uniforms(uint32_t seed, int64_t count, double* out) {
    orc_mt st;
    orc_mt_seed(&st, seed);
    for (int64_t i = 0; i < count; i++) out[i] = orc_canonical53(&st);
}

/* ---- the draw ----------------------------------------------------------- */
/* lower_bound's halving loop over cp[0..n): the first i with !(cp[i] < u). */
static int lower_bound_d(const double* cp, int n, double u) {
    int first = 0, len = n;
    while (len > 0) {
        const int half = len >> 1;
        const int middle = first + half;
        if (cp[middle] < u) {
            first = middle + 1;
            len = len - half - 1;
        } else {
            len = half;
        }
    }
    return first;
}

/*
 * One draw of sample_temperature (main.cpp:91-111) whose generator step
 * produced u.  scratch holds n doubles.  Returns the index, or -1 when
 * scratch is missing.
 */
int orc_sample_temperature_u(const float* logits, int n, float temperature, double u,
                             double* scratch) {
    if (temperature <= 0.0f) return orc_argmax_f32(logits, n);
    if (scratch == NULL) return -1;
    float max_val = logits[0];
    for (int i = 1; i < n; i++)
        if (logits[i] > max_val) max_val = logits[i];
    double* p = scratch;
    double sum = 0.0;
    for (int i = 0; i < n; i++) {
        p[i] = exp((double)((logits[i] - max_val) / temperature));
        sum += p[i];
    }
    for (int i = 0; i < n; i++) p[i] /= sum;
    /* discrete_distribution(probs) */
    if (n < 2) return 0;
    double s2 = 0.0;
    for (int i = 0; i < n; i++) s2 = s2 + p[i];
    for (int i = 0; i < n; i++) p[i] = p[i] / s2;
    double acc = p[0];
    for (int i = 1; i < n; i++) {
        acc = acc + p[i];
        p[i] = acc;
    }
    p[n - 1] = 1.0;
    return lower_bound_d(p, n, u);
}

/* ---- row driver ---------------------------------------------------------- */
#include <pthread.h>
#include <stdlib.h>

typedef struct {
    const float* logits;
    const double* u;
    int32_t* out;
    int64_t r0, r1, cols;
    float temperature;
    int rc;
} sample_slice;

static void* sample_rows(void* arg) {
    sample_slice* s = (sample_slice*)arg;
    double* scratch = (double*)malloc((size_t)s->cols * sizeof(double));
    if (scratch == NULL) {
        s->rc = 7; /* TB_ERR_OUT_OF_MEMORY */
        return NULL;
    }
    for (int64_t r = s->r0; r < s->r1; r++)
        s->out[r] = orc_sample_temperature_u(s->logits + r * s->cols, (int)s->cols,
                                             s->temperature, s->u[r], scratch);
    free(scratch);
    return NULL;
}

int orc_rows_sample_temperature(int64_t rows, int64_t cols, const float* logits,
                                float temperature, const double* u, int32_t* out, int nthreads) {
    if (rows < 0 || cols < 1 || cols > 2147483647 || logits == NULL || u == NULL || out == NULL)
        return ORC_ERR_INVALID_ARG;
    if (nthreads < 1) nthreads = 1;
    if (nthreads > rows) nthreads = rows > 0 ? (int)rows : 1;
    sample_slice* sl = (sample_slice*)calloc((size_t)nthreads, sizeof(sample_slice));
    pthread_t* th = (pthread_t*)calloc((size_t)nthreads, sizeof(pthread_t));
    if (sl == NULL || th == NULL) {
        free(sl);
        free(th);
        return 7;
    }
    const int64_t per = (rows + nthreads - 1) / nthreads;
    for (int i = 0; i < nthreads; i++) {
        sl[i] = (sample_slice){logits, u, out, i * per, (i + 1) * per < rows ? (i + 1) * per : rows,
                               cols, temperature, ORC_OK};
        if (sl[i].r0 > sl[i].r1) sl[i].r0 = sl[i].r1;
        if (nthreads == 1)
            sample_rows(&sl[i]);
        else
            pthread_create(&th[i], NULL, sample_rows, &sl[i]);
    }
    int rc = ORC_OK;
    for (int i = 0; i < nthreads; i++) {
        if (nthreads > 1) pthread_join(th[i], NULL);
        if (sl[i].rc) rc = sl[i].rc;
    }
    free(sl);
    free(th);
    return rc;
}
