// k_softmax.cu -- numerically stable row softmax, with the reference's exact
// row sum.
//
// Reference arithmetic (tb_cpu_softmax_f32, src/ops/softmax.c:4-32), per row:
//   v_i   = x_i (+ mask_i)                      (one f32 add when a mask is given)
//   m     = max_i v_i  (strict '>', from -inf: NaN never becomes the max)
//   e_i   = expf(v_i - m);   sum = ((e_0 + e_1) + e_2) + ...   (f32, in order)
//   y_i   = e_i * (1.0f/sum)   if sum > 0,   else y_i = e_i
// The max is exact in any order.  The sum is reproduced bit-for-bit (see
// ordered_sum.cuh for why an in-order f32 sum can be computed with integer
// prefix sums); expf is CUDA's full-precision expf (within 2 ulp of the C
// library's), the only source of difference from the CPU.
//
// One CTA per row (512 threads, two CTAs per SM), the row cut into 256-term
// tiles (32 lanes x 8 terms); each warp keeps kU tiles of loads in flight:
//   pass 1  per-tile max and an approximate per-tile sum of exp(v - tile
//           max) (fast __expf; an estimate only).  Row max m.
//   est     block scan of the rescaled tile sums: an estimate of the running
//           sum at each tile start, hence a predicted binade b_i per tile.
//           Tiles likely to need term-by-term work (the first tile, a
//           predicted binade change, an estimate near a power of two) get a
//           shared-memory slot for their terms.
//   pass 2  e_i = expf(v_i - m) (stored into y for f32 output, and into the
//           tile's slot); per tile the exact integer sum D_i = sum rne(e/u)
//           on the grid of b_i and whether it holds an exact tie (tie tiles
//           take a free slot too).
//   pass 3  warp 0, 32 tiles per step: while the exact running sum is in a
//           tile's predicted binade, the tile holds no tie, and the sum does
//           not cross into the next binade, the tile is consumed in O(1)
//           (S += D_i).  Otherwise -- about log2(V) binade crossings per row
//           plus the rare tie or misprediction, ~5% of the tiles -- it is
//           summed term by term (ordered_sum_tile), from its slot when it
//           has one.  The first tile, where the sum crosses many binades, is
//           one lane's plain f32 additions.  The result is the sequential
//           sum.
//   pass 4  y = e * (1/sum).
// HBM: one read of x, one write of y; the re-reads hit L2 (two rows per SM
// in flight: ~80 MB at V = 32000 f32), helped by evict-first hints on the
// last read of x and streaming stores of y.  Rows wider than the tile table
// (> 2.8M terms) use one warp for the whole ordered sum.
#include <math.h>

#include "ordered_sum.cuh"
#include "tb_device.cuh"
#include "tb_internal.h"

namespace {

using tbk::Elt;

constexpr int kK = 8;            // terms per lane per tile
constexpr int kTile = 32 * kK;   // terms per tile
constexpr int kTileBytes = 11;   // shared bytes per tile (see k_softmax_tiles)
constexpr int kSlots = 24;       // tiles whose terms are kept in shared memory
constexpr int kNoSlot = 255;
constexpr int kU = 2;            // tiles a warp has in flight

enum Cache { kKeep = 0, kLast = 1 };

template <int CACHE>
__device__ __forceinline__ float4 ld4(const float* p) {
    if constexpr (CACHE == kLast) return __ldcs(reinterpret_cast<const float4*>(p));
    return *reinterpret_cast<const float4*>(p);
}
template <int CACHE>
__device__ __forceinline__ uint4 ld8(const __nv_bfloat16* p) {
    if constexpr (CACHE == kLast) return __ldcs(reinterpret_cast<const uint4*>(p));
    return *reinterpret_cast<const uint4*>(p);
}

// v = x (+ mask) of the kK terms a lane owns in `tile`; missing terms -> -inf.
// VEC: the row is a whole number of 8-term groups and 16-byte aligned, so a
// lane's eight terms are two 16-byte accesses (f32) or one (bf16).
template <typename T, bool VEC, int CACHE = kKeep>
__device__ __forceinline__ int load_oct(const T* xr, const T* mr, int64_t cols, int64_t tile,
                                        int lane, float (&v)[kK]) {
    const int64_t i0 = tile * kTile + lane * kK;
    const int64_t rem = cols - i0;
    const int nv = rem <= 0 ? 0 : (rem >= kK ? kK : (int)rem);
    if (VEC && nv == kK) {
        if constexpr (sizeof(T) == 4) {
            const float4 a = ld4<CACHE>(xr + i0), b = ld4<CACHE>(xr + i0 + 4);
            v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
            v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
            if (mr) {
                const float4 c = ld4<CACHE>(mr + i0), d = ld4<CACHE>(mr + i0 + 4);
                v[0] = __fadd_rn(v[0], c.x); v[1] = __fadd_rn(v[1], c.y);
                v[2] = __fadd_rn(v[2], c.z); v[3] = __fadd_rn(v[3], c.w);
                v[4] = __fadd_rn(v[4], d.x); v[5] = __fadd_rn(v[5], d.y);
                v[6] = __fadd_rn(v[6], d.z); v[7] = __fadd_rn(v[7], d.w);
            }
        } else {
            const uint4 a = ld8<CACHE>(xr + i0);
            const uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                v[2 * q] = __uint_as_float(w[q] << 16);
                v[2 * q + 1] = __uint_as_float(w[q] & 0xffff0000u);
            }
            if (mr) {
                const uint4 c = ld8<CACHE>(mr + i0);
                const uint32_t z[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    v[2 * q] = __fadd_rn(v[2 * q], __uint_as_float(z[q] << 16));
                    v[2 * q + 1] = __fadd_rn(v[2 * q + 1], __uint_as_float(z[q] & 0xffff0000u));
                }
            }
        }
        return kK;
    }
#pragma unroll
    for (int j = 0; j < kK; ++j) {
        v[j] = -INFINITY;
        if (j < nv) {
            v[j] = Elt<T>::load(xr + i0 + j);
            if (mr) v[j] = __fadd_rn(v[j], Elt<T>::load(mr + i0 + j));
        }
    }
    return nv;
}

// Integer grid units of one tile on the FMA pipe.  For t = e/u < 2^22,
// (t + 1.5*2^23) - 1.5*2^23 is t rounded to the nearest integer (the add
// rounds at the units place); |t - r| == 0.5 is an exact tie (its rounding
// depends on the running sum's parity); the units add exactly in f32 while
// the partial sums stay below 2^24, and a tile whose sum reaches 2^24 is an
// event anyway (the running sum leaves its binade).  t >= 2^22 or NaN is an
// event.  Returns the lane's sum; *ev collects the events.
template <int N>
__device__ __forceinline__ float tile_units(const float (&e)[N], int nv, float inv_u, bool* ev) {
    constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23
    float acc = 0.0f;
    bool bad = false;
#pragma unroll
    for (int j = 0; j < N; ++j) {
        const float t = __fmul_rn(j < nv ? e[j] : 0.0f, inv_u);
        const float r = __fsub_rn(__fadd_rn(t, kMagic), kMagic);
        bad |= !(t < 4194304.0f) || fabsf(__fsub_rn(t, r)) == 0.5f;
        acc = __fadd_rn(acc, r);
    }
    *ev |= bad;
    return acc;
}


// Within ~2^-10 relative of a power of two: the exact sum may sit on either
// side of the binade edge the estimate sees.
__device__ __forceinline__ bool near_edge(float v) {
    const uint32_t m = __float_as_uint(v) & 0x7fffffu;
    return m < (1u << 13) || m > (1u << 23) - (1u << 13);
}

// Block-wide exclusive scan (NT threads); `carry` holds NT/32 partials.
template <typename V, int NT>
__device__ __forceinline__ V block_excl_scan(V local, V* carry) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    V incl = local;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const V n = __shfl_up_sync(tbk::kFull, incl, o);
        if (lane >= o) incl += n;
    }
    if (lane == 31) carry[warp] = incl;
    __syncthreads();
    V base = 0;
    for (int w = 0; w < warp; ++w) base += carry[w];
    __syncthreads();
    return base + incl - local;
}

template <typename T, int NT, bool VEC>
__global__ void __launch_bounds__(NT, 2)
k_softmax_tiles(const T* x, const T* mask, T* y, int64_t cols, int ntiles) {
    constexpr int NW = NT / 32;
    constexpr bool kStoreE = sizeof(T) == 4;  // f32 output can hold e exactly
    extern __shared__ __align__(16) unsigned char smem[];
    float (*slots)[kTile] = reinterpret_cast<float (*)[kTile]>(smem);   // kSlots tiles of e
    float* tmax = reinterpret_cast<float*>(smem + sizeof(float) * kSlots * kTile);
    float* tsum = tmax + ntiles;                          // pass 1: tile sum estimate
    uint32_t* tD = reinterpret_cast<uint32_t*>(tmax);    // pass 2: D_i (reuses tmax)
    signed char* tbin = reinterpret_cast<signed char*>(tsum + ntiles);  // predicted binade
    unsigned char* tev = reinterpret_cast<unsigned char*>(tbin + ntiles);  // tile is an event
    unsigned char* tslot = tev + ntiles;                  // slot of the tile's terms
    __shared__ float red[NW];
    __shared__ float fcarry[NW];
    __shared__ int icarry[NW];
    __shared__ float row_sum;
    __shared__ int nslots;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t base = (int64_t)blockIdx.x * cols;
    const T* xr = x + base;
    const T* mr = mask ? mask + base : nullptr;
    T* yr = y + base;

    // ---- pass 1: tile max and tile sum estimate
    for (int tb = warp; tb < ntiles; tb += NW * kU) {
        float v[kU][kK];
        int nv[kU];
#pragma unroll
        for (int u = 0; u < kU; ++u) {
            const int t = tb + u * NW;
            nv[u] = t < ntiles ? load_oct<T, VEC>(xr, mr, cols, t, lane, v[u]) : 0;
        }
#pragma unroll
        for (int u = 0; u < kU; ++u) {
            const int t = tb + u * NW;
            if (t >= ntiles) continue;  // warp-uniform
            float tm = -INFINITY;
#pragma unroll
            for (int j = 0; j < kK; ++j) tm = v[u][j] > tm ? v[u][j] : tm;
            tm = tbk::warp_max(tm);
            float ts = 0.0f;
            if (tm > -INFINITY) {
#pragma unroll
                for (int j = 0; j < kK; ++j)
                    if (j < nv[u]) ts += __expf(v[u][j] - tm);
            }
            ts = tbk::warp_sum(ts);
            if (lane == 0) {
                tmax[t] = tm;
                tsum[t] = ts;
            }
        }
    }
    __syncthreads();
    float m = -INFINITY;
    for (int t = threadIdx.x; t < ntiles; t += NT) m = fmaxf(m, tmax[t]);
    m = tbk::block_max(m, red);

    // ---- estimate of the running sum at each tile start -> predicted binade;
    //      slots for the tiles likely to need term-by-term work
    {
        const int per = (ntiles + NT - 1) / NT;
        const int t0 = min((int)threadIdx.x * per, ntiles);
        const int t1 = min(t0 + per, ntiles);
        float local = 0.0f;
        for (int t = t0; t < t1; ++t) {
            const float tm = tmax[t];
            local += tm > -INFINITY ? tsum[t] * __expf(tm - m) : 0.0f;
        }
        float run = block_excl_scan<float, NT>(local, fcarry);
        int likely = 0;
        for (int t = t0; t < t1; ++t) {
            const int b = tbk::binade_of(run);
            const float tm = tmax[t];
            const float nxt = run + (tm > -INFINITY ? tsum[t] * __expf(tm - m) : 0.0f);
            const bool lk = t == 0 || b == tbk::kNoBinade || tbk::binade_of(nxt) != b ||
                            near_edge(run) || near_edge(nxt);
            tbin[t] = (signed char)b;
            tslot[t] = lk ? 1 : 0;
            likely += lk;
            run = nxt;
        }
        int slot = block_excl_scan<int, NT>(likely, icarry);
        for (int t = t0; t < t1; ++t) {
            if (tslot[t]) {
                tslot[t] = slot < kSlots ? (unsigned char)slot : (unsigned char)kNoSlot;
                ++slot;
            } else {
                tslot[t] = kNoSlot;
            }
        }
        if (threadIdx.x == NT - 1) nslots = slot;
    }
    __syncthreads();  // tmax/tsum fully consumed: tD may now overwrite tmax

    // ---- pass 2: e, the integer tile sums and tie flags
    for (int tb = warp; tb < ntiles; tb += NW * kU) {
        float v[kU][kK];
        int nv[kU];
#pragma unroll
        for (int u = 0; u < kU; ++u) {
            const int t = tb + u * NW;
            nv[u] = t < ntiles ? load_oct<T, VEC, kStoreE ? kLast : kKeep>(xr, mr, cols, t, lane,
                                                                            v[u])
                               : 0;
        }
#pragma unroll
        for (int u = 0; u < kU; ++u) {
            const int t = tb + u * NW;
            if (t >= ntiles) continue;  // warp-uniform
            float e[kK];
#pragma unroll
            for (int j = 0; j < kK; ++j) e[j] = j < nv[u] ? expf(__fsub_rn(v[u][j], m)) : 0.0f;
            const int64_t i0 = (int64_t)t * kTile + lane * kK;
            if constexpr (kStoreE) {
                if (VEC && nv[u] == kK) {
                    *reinterpret_cast<float4*>(yr + i0) = make_float4(e[0], e[1], e[2], e[3]);
                    *reinterpret_cast<float4*>(yr + i0 + 4) = make_float4(e[4], e[5], e[6], e[7]);
                } else {
#pragma unroll
                    for (int j = 0; j < kK; ++j)
                        if (j < nv[u]) Elt<T>::store(yr + i0 + j, e[j]);
                }
            }
            const int b = tbin[t];
            bool ev = b == tbk::kNoBinade;
            float dl = 0.0f;
            if (!ev) dl = tile_units<kK>(e, nv[u], tbk::inv_grid(b), &ev);
            const float dsum = tbk::warp_sum(dl);  // exact below 2^24
            ev = __any_sync(tbk::kFull, ev) || !(dsum < 16777216.0f);
            const uint32_t d = ev ? 0u : (uint32_t)dsum;
            int slot = tslot[t];
            if (slot == kNoSlot && ev) {
                int s = 0;
                if (lane == 0) s = atomicAdd(&nslots, 1);
                s = __shfl_sync(tbk::kFull, s, 0);
                if (s < kSlots) {
                    slot = s;
                    if (lane == 0) tslot[t] = (unsigned char)s;
                }
            }
            if (slot != kNoSlot) {
                *reinterpret_cast<float4*>(&slots[slot][lane * kK]) =
                    make_float4(e[0], e[1], e[2], e[3]);
                *reinterpret_cast<float4*>(&slots[slot][lane * kK + 4]) =
                    make_float4(e[4], e[5], e[6], e[7]);
            }
            if (lane == 0) {
                tD[t] = d;
                tev[t] = ev;
            }
        }
    }
    __syncthreads();

    // ---- pass 3: the ordered sum over tiles (warp 0)
    if (warp == 0) {
        tbk::RunSum st;
        // Tile 0 (always slotted): one lane's plain sequential additions.
        {
            const int n0 = cols < kTile ? (int)cols : kTile;
            float s0 = 0.0f;
            if (lane == 0) {
                const float* e0 = slots[tslot[0]];
                for (int i = 0; i < n0; ++i) s0 = __fadd_rn(s0, e0[i]);
            }
            st.set(__shfl_sync(tbk::kFull, s0, 0));
        }
        for (int t0 = 0; t0 < ntiles && !st.nan; t0 += 32) {
            const int cnt = min(32, ntiles - t0);
            int pos = t0 == 0 ? 1 : 0;
            while (pos < cnt && !st.nan) {
                const int t = t0 + lane;
                const bool valid = lane >= pos && lane < cnt;
                bool ok = false;
                uint32_t d = 0;
                if (valid && st.fast && !tev[t] && tbin[t] == st.b) {
                    ok = true;
                    d = tD[t];
                }
                uint32_t incl = d;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const uint32_t n = __shfl_up_sync(tbk::kFull, incl, o);
                    if (lane >= o) incl = min(incl + n, 1u << 30);
                }
                uint32_t excl = __shfl_up_sync(tbk::kFull, incl, 1);
                if (lane == 0) excl = 0;
                const bool ev = valid && (!ok || st.S + excl + d >= (1u << 24));
                const unsigned bal = __ballot_sync(tbk::kFull, ev);
                if (bal == 0) {
                    st.S += __shfl_sync(tbk::kFull, incl, 31);
                    st.s = __fmul_rn((float)st.S, st.u);
                    break;
                }
                const int f = __ffs(bal) - 1;
                const uint32_t pre = __shfl_sync(tbk::kFull, excl, f);
                if (st.fast && pre) {
                    st.S += pre;
                    st.s = __fmul_rn((float)st.S, st.u);
                }
                // term-by-term through tile t0 + f
                const int tile = t0 + f;
                const int64_t i0 = (int64_t)tile * kTile + lane * kK;
                const int64_t rem = cols - i0;
                const int nv = rem <= 0 ? 0 : (rem >= kK ? kK : (int)rem);
                float e[kK];
                const int slot = tslot[tile];
                if (slot != kNoSlot) {
                    const float4 a = *reinterpret_cast<const float4*>(&slots[slot][lane * kK]);
                    const float4 c = *reinterpret_cast<const float4*>(&slots[slot][lane * kK + 4]);
                    e[0] = a.x; e[1] = a.y; e[2] = a.z; e[3] = a.w;
                    e[4] = c.x; e[5] = c.y; e[6] = c.z; e[7] = c.w;
                } else if constexpr (kStoreE) {
#pragma unroll
                    for (int j = 0; j < kK; ++j) e[j] = j < nv ? Elt<T>::load(yr + i0 + j) : 0.0f;
                } else {
                    float v[kK];
                    load_oct<T, VEC>(xr, mr, cols, tile, lane, v);
#pragma unroll
                    for (int j = 0; j < kK; ++j) e[j] = j < nv ? expf(__fsub_rn(v[j], m)) : 0.0f;
                }
                const int64_t left = cols - (int64_t)tile * kTile;
                tbk::ordered_sum_tile<kK>(st, e, left < kTile ? (int)left : kTile);
                pos = f + 1;
            }
        }
        if (lane == 0) row_sum = st.s;
    }
    __syncthreads();

    // ---- pass 4: normalise
    const float sum = row_sum;
    const bool norm = sum > 0.0f;
    const float inv = __fdiv_rn(1.0f, sum);
    if constexpr (kStoreE) {
        if (!norm) return;  // y already holds e (softmax.c:24)
        for (int tb = warp; tb < ntiles; tb += NW * kU) {
            float4 a[kU][2];
#pragma unroll
            for (int u = 0; u < kU; ++u) {
                const int64_t i0 = (int64_t)(tb + u * NW) * kTile + lane * kK;
                if (VEC && i0 + kK <= cols) {
                    a[u][0] = __ldcs(reinterpret_cast<const float4*>(yr + i0));
                    a[u][1] = __ldcs(reinterpret_cast<const float4*>(yr + i0 + 4));
                }
            }
#pragma unroll
            for (int u = 0; u < kU; ++u) {
                const int64_t i0 = (int64_t)(tb + u * NW) * kTile + lane * kK;
                if (VEC && i0 + kK <= cols) {
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        a[u][h].x = __fmul_rn(a[u][h].x, inv); a[u][h].y = __fmul_rn(a[u][h].y, inv);
                        a[u][h].z = __fmul_rn(a[u][h].z, inv); a[u][h].w = __fmul_rn(a[u][h].w, inv);
                        __stcs(reinterpret_cast<float4*>(yr + i0 + 4 * h), a[u][h]);
                    }
                } else {
                    for (int j = 0; j < kK && i0 + j < cols; ++j)
                        Elt<T>::store(yr + i0 + j, __fmul_rn(Elt<T>::load(yr + i0 + j), inv));
                }
            }
        }
    } else {
        for (int tb = warp; tb < ntiles; tb += NW * kU) {
            float v[kU][kK];
            int nv[kU];
#pragma unroll
            for (int u = 0; u < kU; ++u) {
                const int t = tb + u * NW;
                nv[u] = t < ntiles ? load_oct<T, VEC, kLast>(xr, mr, cols, t, lane, v[u]) : 0;
            }
#pragma unroll
            for (int u = 0; u < kU; ++u) {
                const int64_t i0 = (int64_t)(tb + u * NW) * kTile + lane * kK;
#pragma unroll
                for (int j = 0; j < kK; ++j) {
                    const float e = expf(__fsub_rn(v[u][j], m));
                    v[u][j] = norm ? __fmul_rn(e, inv) : e;
                }
                if (VEC && nv[u] == kK) {
                    uint4 o;
                    o.x = tbk::pack_bf16x2(v[u][0], v[u][1]);
                    o.y = tbk::pack_bf16x2(v[u][2], v[u][3]);
                    o.z = tbk::pack_bf16x2(v[u][4], v[u][5]);
                    o.w = tbk::pack_bf16x2(v[u][6], v[u][7]);
                    __stcs(reinterpret_cast<uint4*>(yr + i0), o);
                } else {
                    for (int j = 0; j < nv[u]; ++j) Elt<T>::store(yr + i0 + j, v[u][j]);
                }
            }
        }
    }
}

// Fallback for rows wider than the tile table: one warp runs the ordered
// sum over the whole row.
template <typename T>
__global__ void __launch_bounds__(256)
k_softmax_wide(const T* x, const T* mask, T* y, int64_t cols) {
    __shared__ float red[32];
    __shared__ float row_sum;
    const int64_t base = (int64_t)blockIdx.x * cols;
    const T* xr = x + base;
    const T* mr = mask ? mask + base : nullptr;
    T* yr = y + base;
    float m = -INFINITY;
    for (int64_t i = threadIdx.x; i < cols; i += blockDim.x) {
        float v = Elt<T>::load(xr + i);
        if (mr) v = __fadd_rn(v, Elt<T>::load(mr + i));
        m = v > m ? v : m;
    }
    m = tbk::block_max(m, red);
    if (threadIdx.x < 32) {
        const int lane = threadIdx.x;
        tbk::RunSum st;
        st.set(0.0f);
        for (int64_t t0 = 0; t0 < cols && !st.nan; t0 += kTile) {
            float e[kK];
#pragma unroll
            for (int j = 0; j < kK; ++j) {
                const int64_t i = t0 + lane * kK + j;
                e[j] = 0.0f;
                if (i < cols) {
                    float v = Elt<T>::load(xr + i);
                    if (mr) v = __fadd_rn(v, Elt<T>::load(mr + i));
                    e[j] = expf(__fsub_rn(v, m));
                }
            }
            const int64_t left = cols - t0;
            tbk::ordered_sum_tile<kK>(st, e, left < kTile ? (int)left : kTile);
        }
        if (lane == 0) row_sum = st.s;
    }
    __syncthreads();
    const float sum = row_sum;
    const bool norm = sum > 0.0f;
    const float inv = __fdiv_rn(1.0f, sum);
    for (int64_t i = threadIdx.x; i < cols; i += blockDim.x) {
        float v = Elt<T>::load(xr + i);
        if (mr) v = __fadd_rn(v, Elt<T>::load(mr + i));
        const float e = expf(__fsub_rn(v, m));
        Elt<T>::store(yr + i, norm ? __fmul_rn(e, inv) : e);
    }
}

template <typename T, int NT, bool VEC>
int launch_tiles(const T* x, const T* m, T* y, int64_t rows, int64_t cols, int ntiles,
                 size_t smem, cudaStream_t s) {
    auto kern = k_softmax_tiles<T, NT, VEC>;
    if (smem > 48 * 1024)
        TB_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem));
    kern<<<(unsigned)rows, NT, smem, s>>>(x, m, y, cols, ntiles);
    TB_LAUNCH_CHECK("softmax kernel");
    return TB_OK;
}

template <typename T>
int launch(int64_t rows, int64_t cols, const void* x, const void* mask, void* y, cudaStream_t s) {
    const T* xp = static_cast<const T*>(x);
    const T* mp = static_cast<const T*>(mask);
    T* yp = static_cast<T*>(y);
    const int64_t ntiles = (cols + kTile - 1) / kTile;
    const size_t smem = sizeof(float) * kSlots * kTile + (size_t)ntiles * kTileBytes + 16;
    if (smem > 200 * 1024) {
        k_softmax_wide<T><<<(unsigned)rows, 256, 0, s>>>(xp, mp, yp, cols);
        TB_LAUNCH_CHECK("softmax kernel");
        return TB_OK;
    }
    const bool vec = cols % kK == 0 && tbh::aligned16(x) && tbh::aligned16(y) &&
                     (mask == nullptr || tbh::aligned16(mask));
    const int nt = (int)ntiles;
    if (cols <= 8192) {
        return vec ? launch_tiles<T, 128, true>(xp, mp, yp, rows, cols, nt, smem, s)
                   : launch_tiles<T, 128, false>(xp, mp, yp, rows, cols, nt, smem, s);
    }
    return vec ? launch_tiles<T, 512, true>(xp, mp, yp, rows, cols, nt, smem, s)
               : launch_tiles<T, 512, false>(xp, mp, yp, rows, cols, nt, smem, s);
}

}  // namespace

extern "C" int tb_b200_softmax(int dtype, int64_t rows, int64_t cols, const void* x,
                               const void* mask, void* y, void* stream) {
    if (rows < 0 || cols < 0 || rows > INT32_MAX) return TB_ERR_INVALID_SHAPE;
    if (rows == 0 || cols == 0) return TB_OK;
    if (!x || !y) return TB_ERR_INVALID_ARG;
    cudaStream_t s = tbh::stream_of(stream);
    if (dtype == TB_DTYPE_F32) {
        if (!mask) {
            int rc = 1;
            if (tbh::softmax_use_cluster())
                rc = tbh::softmax_cluster_f32(rows, cols, static_cast<const float*>(x),
                                              static_cast<float*>(y), s);
            if (rc != 1) return rc;
            rc = tbh::softmax_staged_f32(rows, cols, static_cast<const float*>(x),
                                         static_cast<float*>(y), s);
            if (rc != 1) return rc;
        }
        return launch<float>(rows, cols, x, mask, y, s);
    }
    if (dtype == TB_DTYPE_BF16) return launch<__nv_bfloat16>(rows, cols, x, mask, y, s);
    return TB_ERR_UNSUPPORTED_DTYPE;
}
