// k_sample.cu -- temperature sampling of each row of logits, drawing the
// index the reference draws for the same uniform value.
//
// Reference (sample_temperature, src/main.cpp:91-111): temperature <= 0 is
// greedy argmax; otherwise, per row of n logits,
//   max   = logits[0], then strict '>' over the rest;
//   p_i   = exp((double)((logits[i] - max) / temperature))   (f32 sub and
//           div, double exp);
//   the weights are divided by their in-order double sum, handed to
//   libstdc++'s std::discrete_distribution (which divides them by their sum
//   again, takes in-order partial sums cp and sets cp[n-1] = 1.0), and the
//   draw is lower_bound(cp, u) for u = generate_canonical<double, 53> of the
//   mt19937 generator.  Fewer than two logits draw 0.
// The caller passes u per row (the reference's generator is seeded from
// std::random_device, so only u makes two runs comparable); the oracle
// restates the whole path and is pinned to libstdc++ itself.
//
// One CTA of 256 threads per row:
//   1. the row max (fmaxf over non-NaN values -- the reference's max unless
//      logits[0] is NaN, when every weight is NaN);
//   2. thread t sums the weights of its contiguous 1/256 of the row in double
//      (the reference's f32 argument a = (x - max) / temperature, exp in
//      double); a block scan of the 256 sums gives their in-order offsets
//      and S.  A NaN weight makes every
//      normalised weight NaN and libstdc++'s lower_bound over such a table
//      returns 0 (its halving loop only moves right on cp < u);
//   3. the one thread whose part holds u * S walks it: i* = the first index
//      with P_i / S >= u;
//   4. the reference's cp_i differ from the exact P_i / S by at most
//      (3n + 8) * 2^-53 (two in-order sums and partial sums of n terms, three
//      divisions, exp within an ulp), these by less than (n / 256 + 24) *
//      2^-53.  When u lies more than (4n + 64) * 2^-52 from both P_{i*-1} / S
//      and P_{i*} / S, i* is the reference's draw.  The band must be this
//      narrow: u lands within it of some boundary with probability about
//      sum_i min(q_i, 2 * band) over the normalised weights q_i -- ~2e-6 per
//      row for 32000 N(0, 3) logits, ~3 % with f32 weights (band 1e-6);
//   5. otherwise one thread repeats the
//      reference's arithmetic in order in double: the two sums, the divisions
//      and the partial sums up to the first cp >= u.  Only a one-ulp
//      difference between CUDA's and the C library's double exp can then
//      separate the two answers.
// Data: the logits are read from HBM once (max) and again from L2 (sums).
#include <math.h>

#include "tb_device.cuh"
#include "tb_internal.h"

namespace {

constexpr int kNT = 256;
constexpr int kW = kNT / 32;

// The reference's weight, in double (the in-order path).
__device__ __forceinline__ double weight(float x, float m, float t) {
    return exp((double)__fdiv_rn(__fsub_rn(x, m), t));
}

// The reference's arithmetic, one thread, in order (rare path).
__device__ int sequential_draw(const float* xr, int n, float m, float t, double u) {
    double sum = 0.0;
    for (int i = 0; i < n; i++) sum += weight(xr[i], m, t);
    double s2 = 0.0;
    for (int i = 0; i < n; i++) s2 = s2 + weight(xr[i], m, t) / sum;
    double acc = 0.0;
    for (int i = 0; i < n - 1; i++) {
        const double q = (weight(xr[i], m, t) / sum) / s2;
        acc = i == 0 ? q : acc + q;
        if (acc >= u) return i;
    }
    return n - 1;  // cp[n - 1] = 1.0 > u
}

template <bool VEC>
__global__ void __launch_bounds__(kNT) k_sample(const float* x, int64_t cols, float t,
                                                const double* uniforms, int32_t* out) {
    __shared__ float red[kW];
    __shared__ double wsum[kW];
    __shared__ int verdict;  // -1: to be decided
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t row = blockIdx.x;
    const float* xr = x + row * cols;
    const int n = (int)cols;
    const double u = uniforms[row];

    // 1. max
    float mx = -INFINITY;
    if (VEC) {
        const float4* x4 = reinterpret_cast<const float4*>(xr);
        for (int i = threadIdx.x; i < n / 4; i += kNT) {
            const float4 v = x4[i];
            mx = fmaxf(mx, fmaxf(fmaxf(v.x, v.y), fmaxf(v.z, v.w)));
        }
    } else {
        for (int i = threadIdx.x; i < n; i += kNT) mx = fmaxf(mx, xr[i]);
    }
    mx = tbk::warp_max(mx);
    if (lane == 0) red[warp] = mx;
    if (threadIdx.x == 0) verdict = -1;
    __syncthreads();
    float m = red[0];
#pragma unroll
    for (int w = 1; w < kW; ++w) m = fmaxf(m, red[w]);
    if (xr[0] != xr[0]) {  // the reference's max stays NaN: every weight is NaN
        if (threadIdx.x == 0) out[row] = 0;
        return;
    }

    // 2. thread-contiguous parts (a multiple of 4 terms), summed in double
    const int per = ((n + kNT - 1) / kNT + 3) & ~3;
    const int lo = min(n, (int)threadIdx.x * per), hi = min(n, lo + per);
    double s = 0.0;
    if (VEC) {
        const float4* x4 = reinterpret_cast<const float4*>(xr);
        for (int i = lo / 4; i < hi / 4; ++i) {
            const float4 v = x4[i];
            s += (weight(v.x, m, t) + weight(v.y, m, t)) + (weight(v.z, m, t) + weight(v.w, m, t));
        }
    } else {
        for (int i = lo; i < hi; ++i) s += weight(xr[i], m, t);
    }
    // exclusive block scan of the parts' sums, in thread order
    double inc = s;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const double v = __shfl_up_sync(tbk::kFull, inc, o);
        if (lane >= o) inc += v;
    }
    if (lane == 31) wsum[warp] = inc;
    __syncthreads();
    double base = 0.0, S = 0.0;
#pragma unroll
    for (int w = 0; w < kW; ++w) {
        if (w < warp) base += wsum[w];
        S += wsum[w];
    }
    const double off = base + inc - s;  // weights before this part
    if (!(S >= 1.0 && S < INFINITY)) {  // a NaN weight (S >= 1 otherwise: p_max = 1)
        if (threadIdx.x == 0) out[row] = 0;
        return;
    }

    // 3. the part holding the threshold: parts starting below u * S are a
    //    prefix of the threads; the last of them walks its terms
    const int below = __syncthreads_count(lo < hi && off / S < u);
    if ((int)threadIdx.x == below - 1) {
        double carry = off;
        int found = -1;
        double c_star = 0.0, c_prev = off / S;
        for (int i = lo; i < hi; ++i) {
            carry += weight(xr[i], m, t);
            const double c = carry / S;
            if (c >= u) {
                found = i;
                c_star = c;
                break;
            }
            c_prev = c;
        }
        // 4. the band around the decision
        const double delta = (4.0 * n + 64.0) * 2.220446049250313e-16;  // 2^-52
        if (found >= 0) {
            const bool low_ok = found == 0 || u - c_prev > delta;
            const bool high_ok = found == n - 1 || c_star - u > delta;
            if (low_ok && high_ok) verdict = found;
        }
    }
    __syncthreads();
    if (threadIdx.x != 0) return;
    // 5. close to a boundary (or not found by rounding): the in-order path
    out[row] = verdict >= 0 ? verdict : sequential_draw(xr, n, m, t, u);
}

}  // namespace

extern "C" int tb_b200_sample_temperature(int64_t rows, int64_t cols, const float* logits,
                                          float temperature, const double* uniforms,
                                          int32_t* out, void* stream) {
    if (rows < 0 || cols < 0 || rows > INT32_MAX || cols > INT32_MAX) return TB_ERR_INVALID_SHAPE;
    if (rows == 0) return TB_OK;
    if (cols == 0) return TB_ERR_INVALID_SHAPE;  // the reference reads logits[0]
    if (!logits || !out) return TB_ERR_INVALID_ARG;
    if (temperature <= 0.0f)  // sample_argmax (main.cpp:92)
        return tb_b200_argmax(TB_DTYPE_F32, rows, cols, logits, out, stream);
    cudaStream_t s = tbh::stream_of(stream);
    if (cols < 2) {  // discrete_distribution over one weight draws 0
        TB_CUDA_TRY(cudaMemsetAsync(out, 0, (size_t)rows * sizeof(int32_t), s));
        return TB_OK;
    }
    if (!uniforms) return TB_ERR_INVALID_ARG;
    if (cols % 4 == 0 && tbh::aligned16(logits))
        k_sample<true><<<(unsigned)rows, kNT, 0, s>>>(logits, cols, temperature, uniforms, out);
    else
        k_sample<false><<<(unsigned)rows, kNT, 0, s>>>(logits, cols, temperature, uniforms, out);
    TB_LAUNCH_CHECK("temperature sampling kernel");
    return TB_OK;
}
