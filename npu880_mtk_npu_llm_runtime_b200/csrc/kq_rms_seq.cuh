// kq_rms_seq.cuh -- the sequential fp32 sum of squares of one row, computed by a few dozen
// threads of a CTA at once, bit for bit equal to adding the squares one after another in index
// order (the reference's scalar RMSNorm branch, ENG:4291-4299).
//
// Method (shift-invariant segment chains).  The row is cut into nseg segments.  While a running
// fp32 sum stays in one binade [2^e, 2^(e+1)) every add rounds to the same grid of ulp u, so two
// starts that differ by an even number of ulps give sums that differ by exactly that amount at
// every step (ties to even see the same parity).  After one crossing into the next binade the
// grid is 2u, and starts that differ by a multiple of 4u stay exactly that far apart, provided
// both sums cross at the same add.  So for every segment j >= 1 four threads add the segment from
// c_r = (estimate of the running sum at its start, fp32 bits, low two bits cleared) | r,
// r = 0..3, and each turns its chain into a descriptor {A, B, K, sh}: for every true start S
// (fp32 bits) with S == c_r (mod 4) and A <= S < B, the true sum at the segment's end is
// K + (S >> sh).  The intervals encode the conditions that make the shift exact: S and the chain
// in the same binade, no crossing or exactly one crossing reached at the same add by both sums
// (the crossing add's value and the last value before it are recorded), the end in the binade
// the chain ended in.  Any other chain (two crossings, a non-finite sum, subnormal starts)
// gives the descriptor of its own start only (A = c_r, B = c_r + 1).  Thread 0 adds segment 0
// from 0 and then walks the segments: per segment one descriptor lookup and an add, or, when S
// lies outside the interval, the segment's adds themselves.  Every step is exact, so the result
// is the sequential sum whatever the data; the estimates only decide how often the walk adds a
// segment itself (N(0,1) rows of 2,560 values: ~0.06 segments per row).
//
// Squares of fp16 values are exact in fp32 (11 significant bits -> 22), and they are >= 0, so
// the running sum never decreases: a chain that ends in the binade it started in never left it.
#pragma once

#include "kq_common.cuh"

namespace kq {

constexpr int RMS_MAX_SEG = 32;
// threads of the group: warp 0 runs segment 0 and the walk, warps 1.. the descriptor chains
constexpr int RMS_MIN_THREADS = (32 + 4 * (RMS_MAX_SEG - 1) + 31) / 32 * 32;

struct RmsSegs {
    int L;     // values per segment (a multiple of 128)
    int nseg;  // <= RMS_MAX_SEG
};

__device__ __forceinline__ RmsSegs rms_segments(int K) {
    const int nh = K / 128;
    const int per = (nh + RMS_MAX_SEG - 1) / RMS_MAX_SEG;
    RmsSegs s;
    s.L = 128 * per;
    s.nseg = (nh + per - 1) / per;
    return s;
}

// squares i .. i+3 (i a multiple of 4) of the staged row: staged fp32 squares ...
struct RmsSqF32 {
    const float *sq;
    __device__ __forceinline__ float4 operator()(int i) const { return *reinterpret_cast<const float4 *>(sq + i); }
};
// ... or the staged fp16 values, squared here (exact)
struct RmsSqF16 {
    const __half *xs;
    __device__ __forceinline__ float4 operator()(int i) const {
        const uint2 raw = *reinterpret_cast<const uint2 *>(xs + i);
        const float2 a = __half22float2(*reinterpret_cast<const __half2 *>(&raw.x));
        const float2 b = __half22float2(*reinterpret_cast<const __half2 *>(&raw.y));
        return make_float4(__fmul_rn(a.x, a.x), __fmul_rn(a.y, a.y), __fmul_rn(b.x, b.x), __fmul_rn(b.y, b.y));
    }
};

// Sequential fp32 sum of squares [a, b) (multiples of 32) starting from s.
template <class Q>
__device__ __forceinline__ float rms_chain(const Q &q, int a, int b, float s) {
    for (int i = a; i < b; i += 32) {
        float4 v[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) v[k] = q(i + 4 * k);  // all loads first, then the dependent adds
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            s = __fadd_rn(s, v[k].x);
            s = __fadd_rn(s, v[k].y);
            s = __fadd_rn(s, v[k].z);
            s = __fadd_rn(s, v[k].w);
        }
    }
    return s;
}

// The chain of segment [a, b) from start bits c, as a descriptor {A, B, K, sh}.
template <class Q>
__device__ __forceinline__ uint4 rms_chain_desc(const Q &q, int a, int b, uint32_t c) {
    float s = __uint_as_float(c);
    uint32_t ex = c >> 23;  // binade of the running sum at the last group boundary
    int gi = -1, nx = 0;
    uint32_t gpre = 0;
    for (int i = a; i < b; i += 32) {
        float4 v[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) v[k] = q(i + 4 * k);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const float s0 = s;
            s = __fadd_rn(s, v[k].x);
            s = __fadd_rn(s, v[k].y);
            s = __fadd_rn(s, v[k].z);
            s = __fadd_rn(s, v[k].w);
            const uint32_t e1 = __float_as_uint(s) >> 23;
            if (e1 != ex) {
                if (gi < 0) {
                    gi = i + 4 * k;
                    gpre = __float_as_uint(s0);
                }
                nx += (int)(e1 - ex);  // binades crossed (the sum never decreases)
                ex = e1;
            }
        }
    }
    const uint32_t end = __float_as_uint(s);
    const uint32_t e = c >> 23;
    uint4 d = make_uint4(c, c + 1u, end - c, 0u);  // this start only: K + S = end
    if (e == 0u || e >= 253u || (end >> 23) >= 255u) return d;
    const long long E0 = (long long)e << 23, E1 = (long long)(e + 1) << 23, E2 = (long long)(e + 2) << 23;
    if (nx == 0) {
        // one binade: S -> S + (end - c) for S in binade e with the end still in it
        d.x = (uint32_t)E0;
        d.y = (uint32_t)(E1 - (long long)(end - c));
        d.z = end - c;
        d.w = 0u;
        return d;
    }
    if (nx != 1) return d;
    // one crossing: find its add inside group gi (the first group whose binade changed)
    float t = __uint_as_float(gpre);
    uint32_t pre = 0u;
    float add = 0.0f;
    int n1 = 0;
    const float4 v = q(gi);
    const float vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const float u = __fadd_rn(t, vv[k]);
        if ((__float_as_uint(u) >> 23) != (__float_as_uint(t) >> 23)) {
            if (n1 == 0) {
                pre = __float_as_uint(t);
                add = vv[k];
            }
            ++n1;
        }
        t = u;
    }
    if (n1 != 1 || (pre >> 23) != e) return d;
    // The shifted sum (delta = S - c, a multiple of 4 ulps of binade e) crosses at the same add
    // when its last value before it, pre + delta, is still in binade e and pre + delta + add >=
    // 2^(e+1) exactly, i.e. pre + delta >= T, the smallest binade-e value with that property.
    const double two_e1 = __longlong_as_double((long long)(e + 1 - 127 + 1023) << 52);
    const double two_e = __longlong_as_double((long long)(e - 127 + 1023) << 52);
    const double g = two_e1 - (double)add;  // exact: add >= ulp(e) / 2
    const long long T = (g <= two_e) ? E0 : (long long)__float_as_uint(__double2float_ru(g));
    const long long C = c, P = pre, En = end;
    long long A = E0, B = E1;
    A = max(A, C + T - P);          // the crossing add reaches 2^(e+1)
    A = max(A, C - 2 * (En - E1));  // the end stays >= 2^(e+1)
    B = min(B, C + E1 - P);         // no earlier crossing
    B = min(B, C + 2 * (E2 - En));  // the end stays below 2^(e+2)
    if (A >= B) return d;
    // after the crossing one step of binade e+1 is two of binade e: end + (S - c) / 2
    d.x = (uint32_t)A;
    d.y = (uint32_t)B;
    d.z = end - (c >> 1);
    d.w = 1u;
    return d;
}

// The whole sum.  Called by every thread of a group of `threads` threads (whole warps, at least
// RMS_MIN_THREADS); `sync()` synchronises exactly that group.
//  hsum: K / 128 fp32 estimates (sums of 128 consecutive squares in any order), in shared memory
//  desc: RMS_MAX_SEG * 4 uint4 of shared memory
// Thread 0 adds segment 0, warp 0 walks; thread 32 + 4 (j - 1) + r runs segment j from residue r.
// Returns the sum in thread 0 (the other threads' return value is unspecified).
template <class Q, class Sync>
__device__ __forceinline__ float rms_seq_sum(const Q &q, const float *hsum, uint4 *desc, int K, int tid,
                                             Sync sync) {
    const RmsSegs sg = rms_segments(K);
    float first = 0.0f;
    if (tid == 0) {
        first = rms_chain(q, 0, min(K, sg.L), 0.0f);
    } else if (tid >= 32 && (tid & ~31) < 32 + 4 * (sg.nseg - 1)) {
        // every warp holding descriptor threads computes the segment start estimates itself, all
        // 32 lanes: lane j sums segment j's estimates in fp64, then an inclusive scan over lanes
        const int lane = tid & 31, per = sg.L / 128;
        double ss = 0.0;
        if (lane < sg.nseg)
            for (int h = lane * per; h < min(K / 128, (lane + 1) * per); ++h) ss += (double)hsum[h];
        double inc = ss;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const double y = __shfl_up_sync(0xffffffffu, inc, o);
            if (lane >= o) inc += y;
        }
        const double excl = inc - ss;  // estimate of the running sum at the start of segment `lane`
        const int j = 1 + (tid - 32) / 4, r = (tid - 32) & 3;
        const double est = __shfl_sync(0xffffffffu, excl, min(j, 31));
        if (j < sg.nseg) {
            const uint32_t cb = __float_as_uint(__double2float_rn(est)) & ~3u;
            const int a = j * sg.L, b = min(K, a + sg.L);
            desc[4 * j + r] = rms_chain_desc(q, a, b, cb | (uint32_t)r);
        }
    }
    sync();
    if (tid >= 32) return 0.0f;
    // The walk, by warp 0: lane j holds segment j's four descriptors; at step j every lane maps
    // the current S through its own segment and lane j's result is broadcast.  Lane j records
    // whether S lay in its interval; after the walk one ballot finds the first segment where it
    // did not, and lane 0 continues from there segment by segment.
    const int lane = tid;
    uint4 q0 = make_uint4(0u, 0u, 0u, 0u), q1 = q0, q2 = q0, q3 = q0;
    if (lane >= 1 && lane < sg.nseg) {
        q0 = desc[4 * lane];
        q1 = desc[4 * lane + 1];
        q2 = desc[4 * lane + 2];
        q3 = desc[4 * lane + 3];
    }
    uint32_t S = __shfl_sync(0xffffffffu, __float_as_uint(first), 0);
    uint32_t s_in = 0u;
    bool ok = true;
    for (int j = 1; j < sg.nseg; ++j) {
        const uint32_t r = S & 3u;
        const uint4 lo = (r & 1u) ? q1 : q0, hi = (r & 1u) ? q3 : q2;
        const uint4 d = (r & 2u) ? hi : lo;
        if (lane == j) {
            s_in = S;
            ok = S - d.x < d.y - d.x;
        }
        S = __shfl_sync(0xffffffffu, d.z + (S >> d.w), j);
    }
    const unsigned bad = __ballot_sync(0xffffffffu, !ok);
    if (bad != 0u) {
        // from the first segment whose start fell outside its interval: add it, then continue
        int j = __ffs(bad) - 1;
        S = __shfl_sync(0xffffffffu, s_in, j);
        if (lane != 0) return 0.0f;
        for (; j < sg.nseg; ++j) {
            const uint4 d = desc[4 * j + (S & 3u)];
            if (S - d.x < d.y - d.x) {
                S = d.z + (S >> d.w);
            } else {
                const int a = j * sg.L, b = min(K, a + sg.L);
                S = __float_as_uint(rms_chain(q, a, b, __uint_as_float(S)));
            }
        }
    }
    return __uint_as_float(S);
}

}  // namespace kq
