// k_softmax.cu -- numerically stable row softmax, with the reference's exact
// row sum: rows wider than the staged kernel's (k_softmax_staged.cu), masked
// rows, and bf16.
//
// Reference arithmetic (tb_cpu_softmax_f32, src/ops/softmax.c:4-32), per row:
//   v_i   = x_i (+ mask_i)                      (one f32 add when a mask is given)
//   m     = max_i v_i  (strict '>', from -inf: NaN never becomes the max)
//   e_i   = expf(v_i - m);   sum = ((e_0 + e_1) + e_2) + ...   (f32, in order)
//   y_i   = e_i * (1.0f/sum)   if sum > 0,   else y_i = e_i
// The max is exact in any order.  e_i is tbsm::expo(v_i, m) (ex2-based, the
// same expression as the staged kernel's), and the sum is the in-order f32
// sum of those terms, bit for bit (scan_tiles.cuh).
//
// One CTA per row (512 threads, two CTAs per SM), the row cut into 256-term
// tiles (32 lanes x 8 terms); each warp keeps kU tiles of loads in flight:
//   pass 1  per-tile max and an approximate per-tile sum of exp(v - tile
//           max) (fast __expf; an estimate only).  Row max m.
//   est     block scan of the rescaled tile sums: an estimate of the running
//           sum at each tile start, hence a predicted binade b_t per tile.
//           Tiles likely to need term-by-term work (the first tile, a
//           predicted binade change, an estimate near a power of two) get a
//           shared-memory slot for their terms.
//   pass 2  e_i; per tile the integer sum D
//           of rne(e/u) on the grid of b_t; a tile with an exact tie or a
//           term of 2^22 units or more is flagged (kStop) and takes a free
//           slot.  A slotted tile keeps its terms and the prefix sums of
//           their units on the grids of b_t and b_t + 1 (scan_tiles.cuh,
//           slot tables).  The warp that has tile 0 sums its terms in order.
//   pass 3  warp 0: scan_tiles_tab -- runs of plain tiles added with one
//           redux per 32 tiles, each slotted or flagged tile resolved with
//           a ballot per event over its prefix table, a misprediction
//           located with a scan, a tile without a slot summed term by term
//           (terms recomputed from x).
//   pass 4  y = e * (1/sum), e recomputed from x.
// HBM: one read of x, one write of y; passes 2 and 4 read x again from L2
// (two rows per SM in flight, 152 MB, a little more than L2 holds), helped
// by evict-last hints on pass 1's reads of x, evict-first hints on pass 4's
// (the last), and streaming stores of y.  Pass 2 walks the row from its end,
// passes 1 and 4 from its start: each pass begins with the tiles the one
// before touched last, so the lines L2 has kept longest are not the ones
// needed first.
// e is never stored: a store of e into y and its re-read in pass 4 would
// double the row data each CTA keeps live in L2.  Rows wider than the tile
// table (> 2.7M terms) use one warp for the whole ordered sum.
#include <math.h>

#include <algorithm>

#include "ordered_sum.cuh"
#include "scan_tiles.cuh"
#include "tb_device.cuh"
#include "tb_internal.h"
#include "tma.cuh"

namespace {

using tbk::Elt;
using tbsm::expo;

constexpr int kK = 8;            // terms per lane per tile
constexpr int kTile = 32 * kK;   // terms per tile
static_assert(kTile == tbsm::kTileN, "tile size shared with scan_tiles.cuh");
constexpr int kTileBytes = 12;   // shared bytes per tile (see k_softmax_tiles)
constexpr int kSlots = 24;       // tiles whose terms are kept in shared memory

// L2 policy of a load: default, streaming (last use), or evict-last (f32
// only: pass 1's loads of x, which passes 2 and 4 read again).
enum Cache { kKeep = 0, kLast = 1, kHold = 2 };

template <int CACHE>
__device__ __forceinline__ float4 ld4(const float* p) {
    if constexpr (CACHE == kLast) return __ldcs(reinterpret_cast<const float4*>(p));
    if constexpr (CACHE == kHold)
        return tbk::ld_f4_hint(reinterpret_cast<const float4*>(p), tbk::policy_evict_last());
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

// Terms of a tile without a slot, for the scanner: recomputed from x (+ mask).
template <typename T, bool VEC>
struct RowTerms {
    const T* xr;
    const T* mr;
    int64_t cols;
    float m;
    __device__ __forceinline__ void operator()(int tile, int n, float (&e)[kK]) const {
        const int lane = threadIdx.x & 31;
        float v[kK];
        load_oct<T, VEC>(xr, mr, cols, tile, lane, v);
#pragma unroll
        for (int j = 0; j < kK; ++j) e[j] = lane * kK + j < n ? expo(v[j], m) : 0.0f;
    }
};

// A warp's tiles warp, warp + NW, ... (REV: counted from the row's end) in
// steps of KU tiles, each step's loads issued before the previous step is
// processed (two register sets): load(t, v) fills the lane's kK terms of
// tile t and returns how many are in the row; proc(t, v, nv) may overwrite v.
template <int NW, int KU, bool REV = false, class Load, class Proc>
__device__ __forceinline__ void warp_tiles(int warp, int ntiles, const Load& load,
                                           const Proc& proc) {
    auto at = [&](int t) { return REV ? ntiles - 1 - t : t; };
    float a[KU][kK], b[KU][kK];
    int na[KU], nb[KU];
#pragma unroll
    for (int u = 0; u < KU; ++u) {
        const int t = warp + u * NW;
        na[u] = t < ntiles ? load(at(t), a[u]) : 0;
    }
    for (int tb = warp; tb < ntiles; tb += NW * KU) {
#pragma unroll
        for (int u = 0; u < KU; ++u) {
            const int t = tb + (KU + u) * NW;
            nb[u] = t < ntiles ? load(at(t), b[u]) : 0;
        }
#pragma unroll
        for (int u = 0; u < KU; ++u) {
            const int t = tb + u * NW;
            if (t < ntiles) proc(at(t), a[u], na[u]);  // warp-uniform
        }
#pragma unroll
        for (int u = 0; u < KU; ++u) {
            na[u] = nb[u];
#pragma unroll
            for (int j = 0; j < kK; ++j) a[u][j] = b[u][j];
        }
    }
}

// Max over the warp of lane values that are not NaN: one redux.sync over
// their bits mapped to an order-preserving unsigned key.
__device__ __forceinline__ float warp_max_redux(float v) {
    const uint32_t b = __float_as_uint(v);
    const uint32_t k = __reduce_max_sync(tbk::kFull, (b & 0x80000000u) ? ~b : (b | 0x80000000u));
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

// One row (the whole CTA).  Pass 4 recomputes e from x (the same
// expression, so the same bits): x is the only row-sized data a CTA keeps
// live in L2.
template <typename T, int NT, bool VEC, int KU, int KU2>
__device__ __forceinline__ void tiles_row(const T* x, const T* mask, T* y, int64_t row,
                                          int64_t cols, int ntiles, int nslot) {
    constexpr int NW = NT / 32;
    constexpr int kU = KU;    // tiles per step of a warp in passes 1 and 4
    constexpr int kU2 = KU2;  // the same in pass 2 (more registers per tile)
    extern __shared__ __align__(16) unsigned char smem[];
    tbsm::SlotTab* slots = reinterpret_cast<tbsm::SlotTab*>(smem);  // nslot slotted tiles
    float2* tms = reinterpret_cast<float2*>(smem + sizeof(tbsm::SlotTab) * nslot);
    uint32_t* tD = reinterpret_cast<uint32_t*>(tms);      // pass 2: units per tile, reuses tms
    uint32_t* tmeta = reinterpret_cast<uint32_t*>(tms + ntiles);  // binade | flags | slot << 24
    __shared__ float red[NW];
    __shared__ float fcarry[NW];
    __shared__ int icarry[NW];
    __shared__ float row_sum;
    __shared__ float tile0_sum;
    __shared__ int nslots;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t base = row * cols;
    const T* xr = x + base;
    const T* mr = mask ? mask + base : nullptr;
    T* yr = y + base;

    // ---- pass 1: tile max and tile sum estimate
    warp_tiles<NW, kU>(
        warp, ntiles,
        [&](int t, float (&v)[kK]) { return load_oct<T, VEC, kHold>(xr, mr, cols, t, lane, v); },
        [&](int t, float (&v)[kK], int nv) {
            float tm = -INFINITY;
#pragma unroll
            for (int j = 0; j < kK; ++j) tm = v[j] > tm ? v[j] : tm;
            tm = warp_max_redux(tm);
            float ts = 0.0f;
            if (tm > -INFINITY) {
#pragma unroll
                for (int j = 0; j < kK; ++j)
                    if (j < nv) ts += __expf(v[j] - tm);
            }
            ts = tbsm::warp_sum_est(ts);
            if (lane == 0) tms[t] = make_float2(tm, ts);
        });
    __syncthreads();
    float m = -INFINITY;
    for (int t = threadIdx.x; t < ntiles; t += NT) m = fmaxf(m, tms[t].x);
    m = tbk::block_max(m, red);

    // ---- estimate of the running sum at each tile start -> predicted binade;
    //      slots for the tiles likely to need term-by-term work
    {
        const int per = (ntiles + NT - 1) / NT;
        const int t0 = min((int)threadIdx.x * per, ntiles);
        const int t1 = min(t0 + per, ntiles);
        float local = 0.0f;
        for (int t = t0; t < t1; ++t) {
            const float2 q = tms[t];
            local += q.x > -INFINITY ? q.y * __expf(q.x - m) : 0.0f;
        }
        float run = block_excl_scan<float, NT>(local, fcarry);
        int likely = 0;
        for (int t = t0; t < t1; ++t) {
            const int b = tbk::binade_of(run);
            const float2 q = tms[t];
            const float nxt = run + (q.x > -INFINITY ? q.y * __expf(q.x - m) : 0.0f);
            const bool lk = t == 0 || b == tbk::kNoBinade || tbk::binade_of(nxt) != b ||
                            tbsm::near_pow2(run) || tbsm::near_pow2(nxt);
            tmeta[t] = ((uint32_t)b & 0xffu) | (lk ? (1u << 31) : 0u);
            likely += lk;
            run = nxt;
        }
        int slot = block_excl_scan<int, NT>(likely, icarry);
        for (int t = t0; t < t1; ++t) {
            uint32_t sl = tbsm::kNoSlot;
            if (tmeta[t] >> 31) {
                if (slot < nslot) sl = (uint32_t)slot;
                ++slot;
            }
            tmeta[t] = (tmeta[t] & 0xffu) | (sl << 24);
        }
        if (threadIdx.x == NT - 1) nslots = slot;
    }
    __syncthreads();  // tms fully consumed: tD may now overwrite it

    // ---- pass 2: e, the tiles' units, slots, tile 0's in-order sum
    warp_tiles<NW, kU2, true>(  // last tile first: see the file comment
        warp, ntiles,
        [&](int t, float (&v)[kK]) {
            return load_oct<T, VEC>(xr, mr, cols, t, lane, v);
        },
        [&](int t, float (&e)[kK], int nv) {
#pragma unroll
            for (int j = 0; j < kK; ++j) e[j] = j < nv ? expo(e[j], m) : 0.0f;
            uint32_t meta = tmeta[t];
            const int b = (int)(int8_t)(meta & 0xffu);
            const float iu = tbk::inv_grid(b == tbk::kNoBinade ? 0 : b);
            float acc = 0.0f, dm = 0.0f;
#pragma unroll
            for (int j = 0; j < kK; ++j) {
                const float tt = __fmul_rn(e[j], iu);
                const float r = __fsub_rn(__fadd_rn(tt, tbsm::kMagic), tbsm::kMagic);
                acc = __fadd_rn(acc, r);
                dm = fmaxf(dm, fabsf(__fsub_rn(tt, r)));
            }
            // acc < 2^22 - 1 implies every t < 2^22 - 1/2: the magic rounding
            // was exact; NaN fails the test too.  A tile with an exact tie or
            // such a term is resolved by the scanner (kStop).
            const bool big = __any_sync(tbk::kFull, !(acc < 4194303.0f));
            const bool tie = __any_sync(tbk::kFull, dm == 0.5f);
            const uint32_t d = __reduce_add_sync(
                tbk::kFull, tbsm::magic_int(__fadd_rn(fminf(acc, 4194303.0f), tbsm::kMagic)));
            if (b == tbk::kNoBinade)
                meta |= tbsm::kExact;
            else if (big || tie)
                meta |= tbsm::kStop;
            uint32_t slot = meta >> 24;
            if (slot == tbsm::kNoSlot && (meta & (tbsm::kExact | tbsm::kStop))) {
                int sn = 0;
                if (lane == 0) sn = atomicAdd(&nslots, 1);
                sn = __shfl_sync(tbk::kFull, sn, 0);
                if (sn < nslot) {
                    slot = (uint32_t)sn;
                    meta = (meta & 0x00ffffffu) | (slot << 24);
                }
            }
            if (slot != tbsm::kNoSlot)
                tbsm::slot_tab_fill(slots[slot], e, (meta & tbsm::kExact) ? tbk::kNoBinade : b);
            if (t == 0) {  // tile 0 (always slotted): one lane's in-order additions
                __syncwarp();
                if (lane == 0) {
                    const float* e0 = slots[slot].e;
                    const int n0 = cols < kTile ? (int)cols : kTile;
                    float s0 = 0.0f;
                    for (int q = 0; q < n0; ++q) s0 = __fadd_rn(s0, e0[q]);
                    tile0_sum = s0;
                }
            }
            if (lane == 0) {
                tD[t] = d;
                tmeta[t] = meta;
            }
        });
    __syncthreads();

    // ---- pass 3: the ordered sum over tiles (warp 0)
    if (warp == 0) {
        const float s = tbsm::scan_tiles_tab(tD, tmeta, tile0_sum, slots, nslot,
                                             RowTerms<T, VEC>{xr, mr, cols, m},
                                             (int)cols);
        if (lane == 0) row_sum = s;
    }
    __syncthreads();

    // ---- pass 4: normalise
    const float sum = row_sum;
    const bool norm = sum > 0.0f;
    const float inv = __fdiv_rn(1.0f, sum);
    {
        warp_tiles<NW, kU>(
            warp, ntiles,
            [&](int t, float (&v)[kK]) { return load_oct<T, VEC, kLast>(xr, mr, cols, t, lane, v); },
            [&](int t, float (&v)[kK], int nv) {
                const int64_t i0 = (int64_t)t * kTile + lane * kK;
#pragma unroll
                for (int j = 0; j < kK; ++j) {
                    const float e = expo(v[j], m);
                    v[j] = norm ? __fmul_rn(e, inv) : e;
                }
                if (VEC && nv == kK) {
                    if constexpr (sizeof(T) == 4) {
                        __stcs(reinterpret_cast<float4*>(yr + i0),
                               make_float4(v[0], v[1], v[2], v[3]));
                        __stcs(reinterpret_cast<float4*>(yr + i0 + 4),
                               make_float4(v[4], v[5], v[6], v[7]));
                    } else {
                        uint4 o;
                        o.x = tbk::pack_bf16x2(v[0], v[1]);
                        o.y = tbk::pack_bf16x2(v[2], v[3]);
                        o.z = tbk::pack_bf16x2(v[4], v[5]);
                        o.w = tbk::pack_bf16x2(v[6], v[7]);
                        __stcs(reinterpret_cast<uint4*>(yr + i0), o);
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < kK; ++j)
                        if (j < nv) Elt<T>::store(yr + i0 + j, v[j]);
                }
            });
    }
}

// Row blockIdx.x.  (A persistent form looping over rows made the compiler
// spill the row's working set to local memory.)
template <typename T, int NT, bool VEC, int KU, int KU2>
__global__ void __launch_bounds__(NT, 2)
k_softmax_tiles(const T* x, const T* mask, T* y, int64_t cols, int ntiles, int nslot) {
    tiles_row<T, NT, VEC, KU, KU2>(x, mask, y, blockIdx.x, cols, ntiles, nslot);
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
                    e[j] = expo(v, m);
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
        const float e = expo(v, m);
        Elt<T>::store(yr + i, norm ? __fmul_rn(e, inv) : e);
    }
}

template <typename T, int NT, bool VEC, int KU = 2, int KU2 = 1>
int launch_tiles(const T* x, const T* m, T* y, int64_t rows, int64_t cols, int ntiles, int nslot,
                 size_t smem, cudaStream_t s) {
    auto kern = k_softmax_tiles<T, NT, VEC, KU, KU2>;
    if (smem > 48 * 1024)
        TB_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem));
    kern<<<(unsigned)rows, NT, smem, s>>>(x, m, y, cols, ntiles, nslot);
    TB_LAUNCH_CHECK("softmax kernel");
    return TB_OK;
}

template <typename T>
int launch(int64_t rows, int64_t cols, const void* x, const void* mask, void* y, cudaStream_t s) {
    const T* xp = static_cast<const T*>(x);
    const T* mp = static_cast<const T*>(mask);
    T* yp = static_cast<T*>(y);
    const int64_t ntiles = (cols + kTile - 1) / kTile;
    // slots for about one tile in four, at least 8 (a short row's crossings
    // are few), at most kSlots
    const int nslot = (int)std::min<int64_t>(ntiles, std::max<int64_t>(8, std::min<int64_t>(kSlots, ntiles / 4)));
    const size_t smem = sizeof(tbsm::SlotTab) * nslot + (size_t)ntiles * kTileBytes + 16;
    if (smem > 200 * 1024) {
        k_softmax_wide<T><<<(unsigned)rows, 256, 0, s>>>(xp, mp, yp, cols);
        TB_LAUNCH_CHECK("softmax kernel");
        return TB_OK;
    }
    const bool vec = cols % kK == 0 && tbh::aligned16(x) && tbh::aligned16(y) &&
                     (mask == nullptr || tbh::aligned16(mask));
    const int nt = (int)ntiles;
    if (cols <= 8192) {
        return vec ? launch_tiles<T, 128, true>(xp, mp, yp, rows, cols, nt, nslot, smem, s)
                   : launch_tiles<T, 128, false>(xp, mp, yp, rows, cols, nt, nslot, smem, s);
    }
    return vec ? launch_tiles<T, 512, true>(xp, mp, yp, rows, cols, nt, nslot, smem, s)
               : launch_tiles<T, 512, false>(xp, mp, yp, rows, cols, nt, nslot, smem, s);
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
