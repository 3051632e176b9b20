// scan_tiles.cuh -- the reference's in-order f32 softmax sum from per-tile
// summaries, shared by the staged (rows up to 32768 terms) and tiled (wider
// rows) softmax kernels.
//
// Reference (tb_cpu_softmax_f32, src/ops/softmax.c:15-22):
//   sum = fl(sum + e_0); sum = fl(sum + e_1); ...   (f32, in index order)
// ordered_sum.cuh gives the integer-grid argument: while the running sum s
// stays in the binade [2^b, 2^(b+1)), s = S*u with u = 2^(b-23) and
// fl(s + e) = (S + rne(e/u))*u, except for exact ties (e/u = k + 1/2, rounded
// to the even result, so dependent on the parity of S).
//
// The producer cuts a row into 256-term tiles and, from an estimate of the
// running sum at each tile start, predicts the binade b_t the exact sum will
// be in there.  Per tile it writes
//   D[t]    = (D0, D1): the integer sum of the tile's units on the grid of
//             b_t, for an even / odd running sum at the tile start (they
//             differ only when a term is an exact tie); (kSat, kSat) when a
//             term's units could not be summed exactly (>= 2^22, NaN);
//   meta[t] = b_t (int8) | kExact (sum the tile term by term) | slot << 24,
// and keeps the terms of the tiles likely to need term-by-term work (a
// predicted binade change, an estimate near a power of two) in slots.
//
// scan_tiles() walks 32 tiles per warp step: an ordered composition scan of
// the (D0, D1) functions gives every tile's exact start; the first tile that
// is not on the current grid, is flagged, or takes the sum to 2^24 units is
// resolved -- a slotted tile by prefix sums of its grid units and a ballot
// (the crossing term is one real f32 addition, the rest of the tile O(1) on
// the next grid), anything else term by term (ordered_sum_tile).  The result
// is the sequential sum, bit for bit, whatever the predictions were: a wrong
// one only costs a term-by-term tile.
#pragma once

#include "ordered_sum.cuh"
#include "tb_device.cuh"

namespace tbsm {

constexpr int kTileN = 256;
constexpr uint32_t kSat = 1u << 30;    // saturation of unit sums
constexpr uint32_t kLimit = 1u << 24;  // S reaching this leaves the binade
constexpr uint32_t kExact = 1u << 16;  // meta flag: sum the tile term by term
constexpr uint32_t kNoSlot = 0xffu;
constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23

// The terms of a slotted tile, in index order.
struct Slot {
    float e[kTileN];
};

// e = 2^((x - m) * log2(e)) on the MUFU pipe (subnormal results flush to 0):
// at most 2 + 1.173|x - m| ulp from exp, which weighted by e itself stays
// below 4e-7 of the row's largest term.  Every pass of a row uses this one
// expression, so every pass sees the same bits.
__device__ __forceinline__ float expo(float x, float m) {
    float r;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(__fmul_rn(__fsub_rn(x, m), 1.44269504f)));
    return r;
}

// Sum over the warp of nonnegative lane values v, to about 2^-21 relative:
// the largest lane value sets a power-of-two scale, each lane rounds
// v * scale to an integer, and one redux.sync adds them.
__device__ __forceinline__ float warp_sum_est(float v) {
    const uint32_t mx = __reduce_max_sync(tbk::kFull, __float_as_uint(v));  // v >= 0: bits order
    if (mx == 0u) return 0.0f;
    if (mx >= 0x7f800000u) return __uint_as_float(0x7fc00000u);  // inf or NaN
    const int ex = (int)(mx >> 23) - 127;                 // largest lane value in [2^ex, 2^(ex+1))
    const int sh = 25 - ex;                               // lane values < 2^26 after scaling
    if (sh > 126) return 0.0f;                            // below 2^-100: no binade anyway
    const float sc = __uint_as_float((uint32_t)(sh + 127) << 23);
    const uint32_t q = __float2uint_rn(__fmul_rn(v, sc));
    const uint32_t tot = __reduce_add_sync(tbk::kFull, q);  // < 32 * 2^26 = 2^31
    return __fmul_rn((float)tot, __uint_as_float((uint32_t)(127 - sh) << 23));
}

// Within ~2^-10 relative of a power of two: the exact sum may sit on either
// side of the binade edge the estimate sees.
__device__ __forceinline__ bool near_pow2(float v) {
    const uint32_t mant = __float_as_uint(v) & 0x7fffffu;
    return mant < (1u << 13) || mant > (1u << 23) - (1u << 13);
}

// For a = t + 1.5*2^23 with 0 <= t < 2^22: rne(t) as an integer, read from
// a's mantissa bits (an integer op instead of a float-to-int conversion).
__device__ __forceinline__ uint32_t magic_int(float a) { return __float_as_uint(a) - 0x4B400000u; }

// Grid units of one term on grid inv_u, exact for any t (slot arrays):
// base = rne(t), or floor(t) for an exact tie; 2^25 (certainly an event)
// for t >= 2^25 or NaN.
__device__ __forceinline__ uint32_t units_exact(float e, float inv_u, bool* tie) {
    const float t = __fmul_rn(e, inv_u);
    if (t < 4194304.0f) {
        const float a = __fadd_rn(t, kMagic);
        const float d = __fsub_rn(t, __fsub_rn(a, kMagic));
        *tie = fabsf(d) == 0.5f;
        return magic_int(a) - (d < 0.0f && *tie ? 1u : 0u);
    }
    *tie = false;
    if (!(t < 33554432.0f)) return 1u << 25;
    const float fl = floorf(t);
    *tie = __fsub_rn(t, fl) == 0.5f;
    return *tie ? (uint32_t)fl : __float2uint_rn(t);
}

// Units added by a run of terms given the parity of the partial sum before it.
struct Fn {
    uint32_t a0, a1;  // total for an even / odd running sum at the start
};
__device__ __forceinline__ Fn compose(Fn f, Fn g) {  // f, then g
    Fn r;
    r.a0 = min(f.a0 + ((f.a0 & 1u) ? g.a1 : g.a0), kSat);
    r.a1 = min(f.a1 + (((f.a1 + 1u) & 1u) ? g.a1 : g.a0), kSat);
    return r;
}
// One term with t = e/u < 2^22.
__device__ __forceinline__ Fn term_fn(float e, float inv_u) {
    const float t = __fmul_rn(e, inv_u);
    const float a = __fadd_rn(t, kMagic);
    const float d = __fsub_rn(t, __fsub_rn(a, kMagic));
    const uint32_t ri = magic_int(a);
    if (fabsf(d) != 0.5f) return Fn{ri, ri};
    const uint32_t base = d < 0.0f ? ri - 1u : ri;  // floor(t)
    // round half to even: the result (start + base + extra) must be even
    return Fn{base + (base & 1u), base + ((base + 1u) & 1u)};
}
// In-order reduction of the lanes' functions (lane 0 first); valid in lane 0.
__device__ __forceinline__ Fn warp_compose(Fn f) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        Fn g;
        g.a0 = __shfl_down_sync(tbk::kFull, f.a0, o);
        g.a1 = __shfl_down_sync(tbk::kFull, f.a1, o);
        if ((lane & (2 * o - 1)) == 0) f = compose(f, g);
    }
    return f;
}

// Saturating inclusive warp scan of u32.
__device__ __forceinline__ uint32_t warp_incl(uint32_t v) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t n = __shfl_up_sync(tbk::kFull, v, o);
        if (lane >= o) v = min(v + n, kSat);
    }
    return v;
}

// Inclusive prefix sums of a slotted tile's grid units on one grid, in
// registers: lane l holds those of terms 4l..4l+3 (pa) and 128+4l..128+4l+3
// (pb), with their tie bits (bits 0-3, 4-7).  Terms past the row are 0.
struct TilePrefix {
    uint32_t pa[4], pb[4];
    uint32_t tie;
};
__device__ __forceinline__ TilePrefix tile_prefix(const Slot* s, float inv_u) {
    const int lane = threadIdx.x & 31;
    const float4 a = *reinterpret_cast<const float4*>(s->e + 4 * lane);
    const float4 c = *reinterpret_cast<const float4*>(s->e + 128 + 4 * lane);
    const float e[8] = {a.x, a.y, a.z, a.w, c.x, c.y, c.z, c.w};
    uint32_t u[8];
    TilePrefix P;
    P.tie = 0;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
        bool tq;
        u[q] = units_exact(e[q], inv_u, &tq);
        P.tie |= (uint32_t)tq << q;
    }
    const uint32_t ha = min(min(u[0] + u[1], kSat) + min(u[2] + u[3], kSat), kSat);
    const uint32_t hb = min(min(u[4] + u[5], kSat) + min(u[6] + u[7], kSat), kSat);
    const uint32_t ia = warp_incl(ha);
    const uint32_t ib = warp_incl(hb);
    const uint32_t tot_a = __shfl_sync(tbk::kFull, ia, 31);
    uint32_t pa = ia - ha, pb = min(tot_a + (ib - hb), kSat);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        pa = min(pa + u[q], kSat);
        P.pa[q] = pa;
        pb = min(pb + u[4 + q], kSat);
        P.pb[q] = pb;
    }
    return P;
}
// The prefix at term q (warp-uniform q in [0, 256)).
__device__ __forceinline__ uint32_t prefix_at(const TilePrefix& P, int q) {
    const int r = q & 3;
    const uint32_t* v = q >= 128 ? P.pb : P.pa;
    const uint32_t x = r == 0 ? v[0] : r == 1 ? v[1] : r == 2 ? v[2] : v[3];
    return __shfl_sync(tbk::kFull, x, (q & 127) >> 2);
}

// Consume `tile` into the running sum, exactly.  A slotted tile on the
// current grid: the prefix arrays of grid b (then b+1 after a crossing) find
// each event -- the first term that is a tie or takes the sum to 2^24 units
// -- which is one real f32 addition; the terms between events add in O(1).
// Anything else: term by term, the terms from the slot or from
// terms(tile, n, e) (lane l: terms 8l .. 8l+7, 0 past n).
template <class Terms>
__device__ __forceinline__ void resolve_tile(tbk::RunSum& st, const Slot* slots, int nslot,
                                             const Terms& terms, int tile, uint32_t meta,
                                             int cols) {
    const int lane = threadIdx.x & 31;
    const int tb = (int)(int8_t)(meta & 0xffu);
    const uint32_t slot = meta >> 24;
    const Slot* s = slot < (uint32_t)nslot ? slots + slot : nullptr;
    const int n = min(kTileN, cols - tile * kTileN);
    int pos = 0;
    if (s && !(meta & kExact) && st.fast && st.b == tb) {
        int gcur = -1;
        TilePrefix P;
        while (pos < n && !st.nan) {
            const int g = st.fast ? st.b - tb : -1;
            if (g != 0 && g != 1) break;
            if (g != gcur) {
                P = tile_prefix(s, tbk::inv_grid(tb + g));
                gcur = g;
            }
            const uint32_t P0 = pos ? prefix_at(P, pos - 1) : 0u;
            uint32_t ea = 0, eb = 0;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int ja = 4 * lane + k, jb = 128 + 4 * lane + k;
                if (ja >= pos && ja < n && (((P.tie >> k) & 1u) || st.S + (P.pa[k] - P0) >= kLimit))
                    ea |= 1u << k;
                if (jb >= pos && jb < n &&
                    (((P.tie >> (4 + k)) & 1u) || st.S + (P.pb[k] - P0) >= kLimit))
                    eb |= 1u << k;
            }
            const unsigned ba = __ballot_sync(tbk::kFull, ea != 0);
            const unsigned bb = __ballot_sync(tbk::kFull, eb != 0);
            if (!ba && !bb) {
                st.S += prefix_at(P, n - 1) - P0;
                st.s = __fmul_rn((float)st.S, st.u);
                return;
            }
            int j;
            if (ba) {
                const int f = __ffs(ba) - 1;
                j = 4 * f + __ffs(__shfl_sync(tbk::kFull, ea, f)) - 1;
            } else {
                const int f = __ffs(bb) - 1;
                j = 128 + 4 * f + __ffs(__shfl_sync(tbk::kFull, eb, f)) - 1;
            }
            const uint32_t before = st.S + (j ? prefix_at(P, j - 1) - P0 : 0u);
            st.set(__fadd_rn(__fmul_rn((float)before, st.u), s->e[j]));
            pos = j + 1;
        }
        if (pos >= n || st.nan) return;
    }
    float e[8];
    if (s) {
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const int j = lane * 8 + k;
            e[k] = j < n ? s->e[j] : 0.0f;
        }
    } else {
        terms(tile, n, e);
    }
    tbk::ordered_sum_tile<8>(st, e, n, pos);
}

// The ordered sum of a row of `cols` terms from its tile summaries; s0 is
// the in-order sum of tile 0's terms.  One warp; every lane returns it.
template <class Terms>
__device__ __forceinline__ float scan_tiles(const uint2* D, const uint32_t* meta, float s0,
                                            const Slot* slots, int nslot, const Terms& terms,
                                            int cols) {
    const int lane = threadIdx.x & 31;
    const int ntiles = (cols + kTileN - 1) / kTileN;
    tbk::RunSum st;
    st.set(s0);
    for (int t0 = 0; t0 < ntiles && !st.nan; t0 += 32) {
        const int cnt = min(32, ntiles - t0);
        uint2 dl = make_uint2(0u, 0u);
        uint32_t mt = 0;
        if (lane < cnt) {
            dl = D[t0 + lane];
            mt = meta[t0 + lane];
        }
        const int tb = (int)(int8_t)(mt & 0xffu);
        int pos = t0 == 0 ? 1 : 0;
        while (pos < cnt && !st.nan) {
            const bool valid = lane >= pos && lane < cnt;
            const bool ok = valid && st.fast && !(mt & kExact) && tb == st.b;
            const Fn f = ok ? Fn{dl.x, dl.y} : Fn{0u, 0u};
            Fn inc = f;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                Fn g;
                g.a0 = __shfl_up_sync(tbk::kFull, inc.a0, o);
                g.a1 = __shfl_up_sync(tbk::kFull, inc.a1, o);
                if (lane >= o) inc = compose(g, inc);
            }
            Fn exc;
            exc.a0 = __shfl_up_sync(tbk::kFull, inc.a0, 1);
            exc.a1 = __shfl_up_sync(tbk::kFull, inc.a1, 1);
            if (lane == 0) exc = Fn{0u, 0u};
            const uint32_t p = st.S & 1u;
            const uint32_t ex = p ? exc.a1 : exc.a0;
            const uint32_t mine = ((p + ex) & 1u) ? f.a1 : f.a0;
            const bool ev = valid && (!ok || st.S + ex + mine >= kLimit);
            const unsigned bal = __ballot_sync(tbk::kFull, ev);
            if (bal == 0) {
                st.S += __shfl_sync(tbk::kFull, p ? inc.a1 : inc.a0, 31);
                st.s = __fmul_rn((float)st.S, st.u);
                break;
            }
            const int fl = __ffs(bal) - 1;
            const uint32_t pre = __shfl_sync(tbk::kFull, ex, fl);
            if (st.fast && pre) {
                st.S += pre;
                st.s = __fmul_rn((float)st.S, st.u);
            }
            resolve_tile(st, slots, nslot, terms, t0 + fl, __shfl_sync(tbk::kFull, mt, fl), cols);
            pos = fl + 1;
        }
    }
    return st.s;
}

}  // namespace tbsm

// ------------------------------------------------------------ slot tables
// A second scanner over the same grid argument, for producers that can
// afford to precompute more per slotted tile (the tiled kernel).  A slotted
// tile keeps, besides its terms, the inclusive prefix sums of their units
// on the grids of its predicted binade b and of b + 1, with the tie bits:
// the scanner then finds each event of the tile (the first tie, or the first
// term taking the sum to 2^24 units) with one ballot over values it loads,
// instead of computing units and scans on its own critical path.
// Tiles are walked 32 at a time: a run of tiles on the current grid without
// flags and without slots is added with one redux; the tile that ends the
// run (slotted, flagged, or on another grid) is resolved.  A run that
// crosses 2^24 units anyway (a misprediction) is located with a scan.
namespace tbsm {

constexpr uint32_t kStop = 1u << 17;  // meta flag: a tie or a term >= 2^22 units

struct SlotTab {
    float e[kTileN];                 // the terms, 0 past the row
    uint32_t p[2][kTileN];           // inclusive prefix of units on grids b, b + 1 (saturating)
    uint32_t tie[2][kTileN / 32];    // tie bit of term j: word j >> 5, bit j & 31
};
static_assert(sizeof(SlotTab) % 16 == 0, "slot tables are read with 16-byte loads");

// Producer side, one warp: lane l holds terms 8l .. 8l+7 (0 past the row).
// With b == kNoBinade only the terms are kept (such a tile is summed term
// by term).
__device__ __forceinline__ void slot_tab_fill(SlotTab& T, const float (&e)[8], int b) {
    const int lane = threadIdx.x & 31;
    *reinterpret_cast<float4*>(T.e + 8 * lane) = make_float4(e[0], e[1], e[2], e[3]);
    *reinterpret_cast<float4*>(T.e + 8 * lane + 4) = make_float4(e[4], e[5], e[6], e[7]);
    if (b == tbk::kNoBinade) return;
#pragma unroll
    for (int g = 0; g < 2; ++g) {
        const float iu = tbk::inv_grid(b + g);
        uint32_t c[8];
        uint32_t tb8 = 0, run = 0;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            bool tk;
            run = min(run + units_exact(e[k], iu, &tk), kSat);
            c[k] = run;
            tb8 |= (uint32_t)tk << k;
        }
        const uint32_t incl = warp_incl(run);
        uint32_t excl = __shfl_up_sync(tbk::kFull, incl, 1);
        if (lane == 0) excl = 0u;
#pragma unroll
        for (int k = 0; k < 8; ++k) c[k] = min(excl + c[k], kSat);
        *reinterpret_cast<uint4*>(T.p[g] + 8 * lane) = make_uint4(c[0], c[1], c[2], c[3]);
        *reinterpret_cast<uint4*>(T.p[g] + 8 * lane + 4) = make_uint4(c[4], c[5], c[6], c[7]);
        const uint32_t w = tb8 | (__shfl_down_sync(tbk::kFull, tb8, 1) << 8) |
                           (__shfl_down_sync(tbk::kFull, tb8, 2) << 16) |
                           (__shfl_down_sync(tbk::kFull, tb8, 3) << 24);
        if ((lane & 3) == 0) T.tie[g][lane >> 2] = w;
    }
}

// Consume `tile` into the running sum, exactly: through its slot tables
// while the running sum is on the grid of b or b + 1, otherwise term by
// term (terms from the slot, or from terms(tile, n, e)).
template <class Terms>
__device__ __forceinline__ void resolve_tab(tbk::RunSum& st, const SlotTab* tabs, int nslot,
                                            const Terms& terms, int tile, uint32_t meta,
                                            int cols) {
    const int lane = threadIdx.x & 31;
    const int tb = (int)(int8_t)(meta & 0xffu);
    const uint32_t slot = meta >> 24;
    const SlotTab* T = slot < (uint32_t)nslot ? tabs + slot : nullptr;
    const int n = min(kTileN, cols - tile * kTileN);
    int pos = 0;
    if (T && !(meta & kExact)) {
        while (pos < n && !st.nan) {
            const int g = st.fast ? st.b - tb : -1;
            if (g != 0 && g != 1) break;
            const uint32_t* p = T->p[g];
            const uint32_t P0 = pos ? p[pos - 1] : 0u;
            if (P0 >= kSat - kLimit) break;  // saturated prefixes: term by term
            const uint4 a = *reinterpret_cast<const uint4*>(p + 8 * lane);
            const uint4 c = *reinterpret_cast<const uint4*>(p + 8 * lane + 4);
            const uint32_t tw = (T->tie[g][lane >> 2] >> (8 * (lane & 3))) & 0xffu;
            const uint32_t pv[8] = {a.x, a.y, a.z, a.w, c.x, c.y, c.z, c.w};
            uint32_t evb = 0;
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const int j = 8 * lane + k;
                if (j >= pos && j < n && (((tw >> k) & 1u) || st.S + (pv[k] - P0) >= kLimit))
                    evb |= 1u << k;
            }
            const unsigned bal = __ballot_sync(tbk::kFull, evb != 0);
            if (!bal) {
                st.S += p[n - 1] - P0;
                st.s = __fmul_rn((float)st.S, st.u);
                return;
            }
            const int f = __ffs(bal) - 1;
            const int j = 8 * f + __ffs(__shfl_sync(tbk::kFull, evb, f)) - 1;
            const uint32_t before = st.S + (j ? p[j - 1] - P0 : 0u);
            st.set(__fadd_rn(__fmul_rn((float)before, st.u), T->e[j]));
            pos = j + 1;
        }
        if (pos >= n || st.nan) return;
    }
    float e[8];
    if (T) {
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const int j = lane * 8 + k;
            e[k] = j < n ? T->e[j] : 0.0f;
        }
    } else {
        terms(tile, n, e);
    }
    tbk::ordered_sum_tile<8>(st, e, n, pos);
}

// The ordered sum of a row from D[t] (the tile's units on the grid of its
// predicted binade, valid when meta carries neither kExact nor kStop) and
// meta[t] (b_t | flags | slot << 24); s0 is the in-order sum of tile 0.
// One warp; every lane returns it.
template <class Terms>
__device__ __forceinline__ float scan_tiles_tab(const uint32_t* D, const uint32_t* meta, float s0,
                                                const SlotTab* tabs, int nslot,
                                                const Terms& terms, int cols) {
    const int lane = threadIdx.x & 31;
    const int ntiles = (cols + kTileN - 1) / kTileN;
    tbk::RunSum st;
    st.set(s0);
    for (int t0 = 0; t0 < ntiles && !st.nan; t0 += 32) {
        const int cnt = min(32, ntiles - t0);
        uint32_t d = 0, mt = 0;
        if (lane < cnt) {
            d = D[t0 + lane];
            mt = meta[t0 + lane];
        }
        const int tb = (int)(int8_t)(mt & 0xffu);
        const bool plain = !(mt & (kExact | kStop)) && (mt >> 24) >= (uint32_t)nslot;
        int pos = t0 == 0 ? 1 : 0;
        while (pos < cnt && !st.nan) {
            const bool valid = lane >= pos && lane < cnt;
            const bool ok = valid && plain && st.fast && tb == st.b;
            const unsigned stop = __ballot_sync(tbk::kFull, valid && !ok);
            const int lim = stop ? __ffs(stop) - 1 : cnt;
            const uint32_t dd = lane >= pos && lane < lim ? min(d, 1u << 25) : 0u;
            const uint32_t tot = __reduce_add_sync(tbk::kFull, dd);  // <= 32 * 2^25
            if (tot == 0u || st.S + tot < kLimit) {
                if (tot) {
                    st.S += tot;
                    st.s = __fmul_rn((float)st.S, st.u);
                }
                if (lim == cnt) break;
                resolve_tab(st, tabs, nslot, terms, t0 + lim, __shfl_sync(tbk::kFull, mt, lim),
                            cols);
                pos = lim + 1;
                continue;
            }
            // The run crosses 2^24 units (the binade was mispredicted): the
            // crossing tile, by an inclusive scan of the run.
            uint32_t incl = dd;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const uint32_t nb = __shfl_up_sync(tbk::kFull, incl, o);
                if (lane >= o) incl += nb;
            }
            const unsigned cr = __ballot_sync(tbk::kFull, lane >= pos && lane < lim &&
                                                              st.S + incl >= kLimit);
            const int f = __ffs(cr) - 1;
            st.S += __shfl_sync(tbk::kFull, incl - dd, f);
            st.s = __fmul_rn((float)st.S, st.u);
            resolve_tab(st, tabs, nslot, terms, t0 + f, __shfl_sync(tbk::kFull, mt, f), cols);
            pos = f + 1;
        }
    }
    return st.s;
}

}  // namespace tbsm
