// pin_sampling.cpp -- the reference's temperature sampling with the real
// libstdc++ <random>, for pinning the oracle's restatement (sampling.c).
//
// TEST INFRASTRUCTURE ONLY.  Built by oracle/Makefile into oracle/_ref/ with
// the host's g++ (the toolchain the reference builds with).  It repeats the
// probability arithmetic of sample_temperature (src/main.cpp:91-111; the
// function is static there) and then draws with std::discrete_distribution
// over a std::mt19937 seeded with `seed` (the reference seeds from
// std::random_device, which no test can reproduce), one draw per row in row
// order -- the library code whose behaviour sampling.c restates.
#include <cmath>
#include <cstdint>
#include <random>
#include <vector>

extern "C" int pin_sample_temperature_rows(const float* logits, int64_t rows, int64_t cols,
                                           float temperature, uint32_t seed, int32_t* out) {
    std::mt19937 rng(seed);
    const int n = (int)cols;
    for (int64_t r = 0; r < rows; ++r) {
        const float* x = logits + r * cols;
        if (temperature <= 0.0f) {  // sample_argmax, main.cpp:79-89
            int best = 0;
            float bv = x[0];
            for (int i = 1; i < n; i++)
                if (x[i] > bv) {
                    bv = x[i];
                    best = i;
                }
            out[r] = best;
            continue;
        }
        float max_val = x[0];
        for (int i = 1; i < n; i++)
            if (x[i] > max_val) max_val = x[i];
        std::vector<double> probs(n);
        double sum = 0.0;
        for (int i = 0; i < n; i++) {
            probs[i] = std::exp((double)((x[i] - max_val) / temperature));
            sum += probs[i];
        }
        for (int i = 0; i < n; i++) probs[i] /= sum;
        std::discrete_distribution<int> dist(probs.begin(), probs.end());
        out[r] = dist(rng);
    }
    return 0;
}

// The first `count` values generate_canonical<double, 53> draws from
// std::mt19937(seed), for pinning the oracle's MT19937 and canonical step.
extern "C" void pin_uniforms(uint32_t seed, int64_t count, double* out) {
    std::mt19937 rng(seed);
    for (int64_t i = 0; i < count; ++i) out[i] = std::generate_canonical<double, 53>(rng);
}
