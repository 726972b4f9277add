// qdot.cuh -- Q4_K / Q6_K / Q8_0 decoding on sm_100a.
//
// Two families of device functions:
//   * exact element dequantisation (the arithmetic of the reference CPU
//     decoders layer_ops.cu:44-105, each product rounded separately), used by
//     bread_dequant and by the alignment-agnostic GEMV;
//   * "lane dots": one lane's share of a super-block row dot product against
//     an activation slice quantised to 16-bit fixed point per 32 values.  The
//     weight side stays exact: per sub-block the reference weight is
//     d*sc*q - dmin*m (Q4_K) or d*sc*(q-32) (Q6_K), so
//         sum_i w_i x_i = d*sc*s_x*SUM(q_i xq_i) - dmin*m*s_x*SUM(xq_i)
//     where xq_i = round(x_i / s_x) and the inner SUMs are exact int32 dot
//     products (dp2a).  The only approximation is x ~= s_x*xq
//     (|error| <= s_x/2 = max|x_group| / 65534); the GEMV adds a second
//     int16 level for groups with outliers (quant32_r_n), taking the error of
//     those groups to max|x_group| / 2^31.
#pragma once
#include <stdint.h>
#include "common.cuh"
#include "ptx.cuh"

namespace bread {

// ---------------------------------------------------------------------------
// exact dequantisation (reference layer_ops.cu:44-105, kernels.cu:251-284)
// ---------------------------------------------------------------------------
__device__ __forceinline__ float h2f_bits(uint16_t b) { return __half2float(__ushort_as_half(b)); }

__device__ __forceinline__ void q4k_scale_min(const uint8_t *s, int j, int &sc, int &m)
{
    if (j < 4) {
        sc = s[j] & 63;
        m = s[j + 4] & 63;
    } else {
        sc = (s[j + 4] & 0x0F) | ((s[j - 4] >> 6) << 4);
        m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}

// Element e (0..255) of a Q4_K block: (d*sc)*q - (dmin*m), no FMA.
__device__ __forceinline__ float q4k_elem_exact(const uint8_t *blk, int e)
{
    const float d = h2f_bits((uint16_t)(blk[0] | (blk[1] << 8)));
    const float dmin = h2f_bits((uint16_t)(blk[2] | (blk[3] << 8)));
    const int grp = e >> 6, sub = (e >> 5) & 1, pos = e & 31;
    int sc, m;
    q4k_scale_min(blk + 4, 2 * grp + sub, sc, m);
    const uint8_t qb = blk[16 + 32 * grp + pos];
    const int q = sub ? (qb >> 4) : (qb & 0xF);
    const float d1 = __fmul_rn(d, (float)sc);
    const float m1 = __fmul_rn(dmin, (float)m);
    return __fsub_rn(__fmul_rn(d1, (float)q), m1);
}

// Element e of a Q6_K block: (d*sc)*(q-32), left to right, no FMA.
__device__ __forceinline__ float q6k_elem_exact(const uint8_t *blk, int e)
{
    const float d = h2f_bits((uint16_t)(blk[208] | (blk[209] << 8)));
    const int half = e >> 7, r = (e >> 5) & 3, l = e & 31;
    const uint8_t *ql = blk + 64 * half, *qh = blk + 128 + 32 * half;
    const int8_t *sc = (const int8_t *)(blk + 192 + 8 * half);
    const uint8_t qlb = ql[l + 32 * (r & 1)];
    const int lo4 = (r >> 1) ? (qlb >> 4) : (qlb & 0xF);
    const int hi2 = (qh[l] >> (2 * r)) & 3;
    const int q = (lo4 | (hi2 << 4)) - 32;
    return __fmul_rn(__fmul_rn(d, (float)sc[l / 16 + 2 * r]), (float)q);
}

// Element e (0..31) of a Q8_0 block: d*q.
__device__ __forceinline__ float q80_elem_exact(const uint8_t *blk, int e)
{
    const float d = h2f_bits((uint16_t)(blk[0] | (blk[1] << 8)));
    return __fmul_rn(d, (float)(int8_t)blk[2 + e]);
}

template <int QT>
__device__ __forceinline__ float elem_exact(const uint8_t *blk, int e)
{
    if (QT == BREAD_QTYPE_Q4_K) return q4k_elem_exact(blk, e);
    if (QT == BREAD_QTYPE_Q6_K) return q6k_elem_exact(blk, e);
    return q80_elem_exact(blk, e);
}

// ---------------------------------------------------------------------------
// activation quantisation: 32 values -> int16 + one fp32 scale
// ---------------------------------------------------------------------------
// Called by a full warp with one value per lane; returns the lane's int16 and
// writes the group scale (max|x| / 32767) to *scale on lane 0.  An all-zero
// group gets scale 0; a non-finite value gives a NaN scale (outputs NaN).
__device__ __forceinline__ int quant32(float v, float *scale, int lane)
{
    float a = fabsf(v);
    // fmaxf drops NaN, so non-finite values are detected separately
    const bool finite = !__any_sync(0xffffffffu, !(a <= 3.402823466e38f));
#pragma unroll
    for (int o = 16; o; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
    int q = 0;
    if (a > 0.0f && finite) q = __float2int_rn((v / a) * 32767.0f);  // |v/a| <= 1, also for subnormal a
    if (lane == 0) *scale = finite ? a * (1.0f / 32767.0f) : __int_as_float(0x7fc00000);
    return q;
}

// quant32 with a second level for a group whose largest value dwarfs the
// rest (outliers, e.g. a massive-activation channel): r quantises the first
// level's error v - q*s to int16 with scale s2, so v ~= q*s + r*s2 with an
// error below s2/2 = max|v| / 2^31.  The first level's rounding error (up to
// s/2, s = max|v|/32767) costs a dot product a relative ~ s / (sqrt(12) *
// rms) of the values it weights; when the weights skip the large values,
// rms is that of the rest.  So a group keeps the second level (s2 > 0) when
// max|v| > 16 * rms of its values below 0.35 max|v| -- where one level would
// cost more than ~1.4e-4 -- which normal or Laplace data meets in ~1e-5 of
// its groups.  Otherwise r = 0, s2 = 0 and q, s are exactly quant32's.
// N groups at once (one value of each per lane, reductions interleaved);
// q, r, s, s2 of group k valid on every lane.
template <int N>
__device__ __forceinline__ void quant32_r_n(const float (&v)[N], int (&q)[N], int (&r)[N], float (&s)[N],
                                            float (&s2)[N])
{
    float a[N], sm[N];
    bool finite[N];
    int n[N];
#pragma unroll
    for (int k = 0; k < N; ++k) {
        a[k] = fabsf(v[k]);
        finite[k] = !__any_sync(0xffffffffu, !(a[k] <= 3.402823466e38f));
    }
#pragma unroll
    for (int o = 16; o; o >>= 1)
#pragma unroll
        for (int k = 0; k < N; ++k) a[k] = fmaxf(a[k], __shfl_xor_sync(0xffffffffu, a[k], o));
#pragma unroll
    for (int k = 0; k < N; ++k) {
        q[k] = (a[k] > 0.0f && finite[k]) ? __float2int_rn((v[k] / a[k]) * 32767.0f) : 0;
        s[k] = finite[k] ? a[k] * (1.0f / 32767.0f) : __int_as_float(0x7fc00000);
        const bool rest = fabsf(v[k]) < 0.35f * a[k];
        n[k] = __popc(__ballot_sync(0xffffffffu, rest));
        sm[k] = rest ? v[k] * v[k] : 0.0f;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1)
#pragma unroll
        for (int k = 0; k < N; ++k) sm[k] += __shfl_xor_sync(0xffffffffu, sm[k], o);
#pragma unroll
    for (int k = 0; k < N; ++k) {
        r[k] = 0;
        s2[k] = 0.0f;
        if (finite[k] && a[k] > 0.0f && a[k] * a[k] * (float)n[k] > 256.0f * sm[k]) {  // (warp-uniform)
            const float e = fmaf(-(float)q[k], s[k], v[k]);
            float b = fabsf(e);
#pragma unroll
            for (int o = 16; o; o >>= 1) b = fmaxf(b, __shfl_xor_sync(0xffffffffu, b, o));
            if (b > 0.0f) {
                r[k] = __float2int_rn((e / b) * 32767.0f);
                s2[k] = b * (1.0f / 32767.0f);
            }
        }
    }
}

// N groups at once (one value of each per lane), the same arithmetic per
// group as quant32, their reductions interleaved: q[k] and the scale sc[k]
// (valid on every lane) of group k.
template <int N>
__device__ __forceinline__ void quant32_n(const float (&v)[N], int (&q)[N], float (&sc)[N])
{
    float a[N];
    bool finite[N];
#pragma unroll
    for (int k = 0; k < N; ++k) {
        a[k] = fabsf(v[k]);
        finite[k] = !__any_sync(0xffffffffu, !(a[k] <= 3.402823466e38f));
    }
#pragma unroll
    for (int o = 16; o; o >>= 1)
#pragma unroll
        for (int k = 0; k < N; ++k) a[k] = fmaxf(a[k], __shfl_xor_sync(0xffffffffu, a[k], o));
#pragma unroll
    for (int k = 0; k < N; ++k) {
        q[k] = (a[k] > 0.0f && finite[k]) ? __float2int_rn((v[k] / a[k]) * 32767.0f) : 0;
        sc[k] = finite[k] ? a[k] * (1.0f / 32767.0f) : __int_as_float(0x7fc00000);
    }
}

// ---------------------------------------------------------------------------
// lane dots
// ---------------------------------------------------------------------------
// Layout of quantised activations (per token, in global and shared memory):
// the eight 16-byte pieces of every 128-byte chunk (64 values) are rotated by
// the chunk index, so value e of the token sits at xq_pos(e).  The lanes of a
// quarter-warp read eight different chunks, piece by piece: with the rotation
// they hit eight different bank groups instead of one.  Positions are
// relative to the token's first value (rows are a multiple of 64 values).
__host__ __device__ __forceinline__ constexpr int xq_pos(int e)
{
    return (e & ~63) | ((((e >> 3) + (e >> 6)) & 7) << 3) | (e & 7);
}
// The 8 values e .. e+7 (e a multiple of 8) of a token stored as above.
__device__ __forceinline__ int4 xq_piece(const int16_t *tok, int e)
{
    return *reinterpret_cast<const int4 *>(tok + xq_pos(e));
}

// One lane's activation slice for one token: 64 int16 (two per int).
struct XSlice {
    int v[32];
    float s[4];
    int c[4];
};

// Q4_K lane (block b, pair g): block elements 64g..64g+63, i.e. sub-blocks 2g
// (low nibbles of qs[32g..32g+31]) and 2g+1 (high nibbles).
// xq/xs: the token's int16 values (xq_pos layout) and per-32 scales;
// e0 = 256*b + 64*g.
// rs multiplies the group scales (the RMS-normalisation factor of the token).
__device__ __forceinline__ void load_slice_q4k(XSlice &X, const int16_t *xq, const float *xs, int e0,
                                               float rs = 1.0f)
{
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int4 t = xq_piece(xq, e0 + 8 * i);
        X.v[4 * i + 0] = t.x;
        X.v[4 * i + 1] = t.y;
        X.v[4 * i + 2] = t.z;
        X.v[4 * i + 3] = t.w;
    }
    int s0 = 0, s1 = 0;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        s0 = sum_i16x2(X.v[i], s0);
        s1 = sum_i16x2(X.v[16 + i], s1);
    }
    const float f0 = xs[e0 >> 5] * rs, f1 = xs[(e0 >> 5) + 1] * rs;
    X.s[0] = f0;
    X.s[1] = f1 * 0.0625f;  // the high nibbles enter the dot product as 16*q
    X.s[2] = f0 * (float)s0;
    X.s[3] = f1 * (float)s1;
}

// blk: 16-byte aligned Q4_K block; g: 0..3.
__device__ __forceinline__ float q4k_lane_dot(const uint8_t *blk, int g, const XSlice &X)
{
    const uint4 hd = *reinterpret_cast<const uint4 *>(blk);
    const uint4 qa = *reinterpret_cast<const uint4 *>(blk + 16 + 32 * g);
    const uint4 qb = *reinterpret_cast<const uint4 *>(blk + 32 + 32 * g);
    const uint32_t w[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
    int p0 = 0, p1 = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const uint32_t lo = w[i] & 0x0F0F0F0Fu, hi = w[i] & 0xF0F0F0F0u;
        p0 = dp2a_lo(X.v[2 * i], lo, p0);
        p0 = dp2a_hi(X.v[2 * i + 1], lo, p0);
        p1 = dp2a_lo(X.v[16 + 2 * i], hi, p1);
        p1 = dp2a_hi(X.v[16 + 2 * i + 1], hi, p1);
    }
    // (scale, min) of sub-blocks 2g and 2g+1 from the 12 packed bytes, both at
    // once (two bytes per field), following dequant_q4k_cpu.c:70-79.
    const uint32_t sh = 16u * (uint32_t)(g & 1);
    const uint32_t A = hd.y >> sh, B = hd.z >> sh, C = hd.w >> sh;
    uint32_t scp, mp;
    if (g >= 2) {
        scp = (C & 0x0F0Fu) | ((A >> 2) & 0x3030u);
        mp = ((C >> 4) & 0x0F0Fu) | ((B >> 2) & 0x3030u);
    } else {
        scp = A & 0x3F3Fu;
        mp = B & 0x3F3Fu;
    }
    const float sc0 = u2f_small(scp & 0xFFu), sc1 = u2f_small((scp >> 8) & 0xFFu);
    const float m0 = u2f_small(mp & 0xFFu), m1 = u2f_small((mp >> 8) & 0xFFu);
    const float2 dd = __half22float2(*reinterpret_cast<const __half2 *>(&hd.x));
    const float u = fmaf(sc1 * X.s[1], (float)p1, (sc0 * X.s[0]) * (float)p0);
    const float mm = fmaf(m1, X.s[3], m0 * X.s[2]);
    return fmaf(dd.x, u, -dd.y * mm);
}

// Q6_K lane (block b, half h, l-group g): block elements 128h + 32r + 16g + i
// for r = 0..3, i = 0..15 (four runs of 16).  base = 256*b + 128*h.
__device__ __forceinline__ void load_slice_q6k(XSlice &X, const int16_t *xq, const float *xs, int base, int g)
{
#pragma unroll
    for (int r = 0; r < 4; ++r) {
        const int4 t0 = xq_piece(xq, base + 32 * r + 16 * g), t1 = xq_piece(xq, base + 32 * r + 16 * g + 8);
        X.v[8 * r + 0] = t0.x;
        X.v[8 * r + 1] = t0.y;
        X.v[8 * r + 2] = t0.z;
        X.v[8 * r + 3] = t0.w;
        X.v[8 * r + 4] = t1.x;
        X.v[8 * r + 5] = t1.y;
        X.v[8 * r + 6] = t1.z;
        X.v[8 * r + 7] = t1.w;
        int s = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) s = sum_i16x2(X.v[8 * r + i], s);
        X.c[r] = 32 * s;
        X.s[r] = xs[(base >> 5) + r];
    }
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel)
{
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}

// 16 bytes at p (2-byte aligned; sh = p & 3, sel = sh ? 0x5432 : 0x3210)
// from 4-byte aligned shared-memory words.
__device__ __forceinline__ void ld16_shift(const uint8_t *p, int sh, uint32_t sel, uint32_t o[4])
{
    const uint32_t *q = reinterpret_cast<const uint32_t *>(p - sh);
    const uint32_t w0 = q[0], w1 = q[1], w2 = q[2], w3 = q[3], w4 = q[4];
    o[0] = prmt(w0, w1, sel);
    o[1] = prmt(w1, w2, sel);
    o[2] = prmt(w2, w3, sel);
    o[3] = prmt(w3, w4, sel);
}

// Per-lane constants of a Q6_K lane: byte shift of its block, permute
// selector, and the four sign-extending selectors picking int8 scales
// g, g+2 (of scales 0..3 of the half) and g, g+2 (of scales 4..7).
struct Q6Lane {
    int sh;
    uint32_t sel;
    uint32_t ssel[2];
};
__device__ __forceinline__ uint32_t sext_sel(int k)
{
    const uint32_t s = (uint32_t)(k | 8);
    return (uint32_t)k | (s << 4) | (s << 8) | (s << 12);
}
__device__ __forceinline__ Q6Lane q6_lane(int sh, int g)
{
    Q6Lane L;
    L.sh = sh;
    L.sel = sh ? 0x5432u : 0x3210u;
    L.ssel[0] = sext_sel(g);
    L.ssel[1] = sext_sel(g + 2);
    return L;
}

// blk: Q6_K block in shared memory (2-byte aligned, (blk & 3) == L.sh).
__device__ __forceinline__ float q6k_lane_dot(const uint8_t *blk, int h, int g, const Q6Lane &L, const XSlice &X)
{
    uint32_t A[4], B[4], Q[4];
    ld16_shift(blk + 64 * h + 16 * g, L.sh, L.sel, A);
    ld16_shift(blk + 64 * h + 32 + 16 * g, L.sh, L.sel, B);
    ld16_shift(blk + 128 + 32 * h + 16 * g, L.sh, L.sel, Q);
    int p0 = 0, p1 = 0, p2 = 0, p3 = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        // 6-bit values of l = 16g+4i..+3 for runs r = 0..3 (dequant_q4k_cpu.c:157-160)
        const uint32_t v0 = (A[i] & 0x0F0F0F0Fu) | ((Q[i] << 4) & 0x30303030u);
        const uint32_t v1 = (B[i] & 0x0F0F0F0Fu) | ((Q[i] << 2) & 0x30303030u);
        const uint32_t v2 = ((A[i] >> 4) & 0x0F0F0F0Fu) | (Q[i] & 0x30303030u);
        const uint32_t v3 = ((B[i] >> 4) & 0x0F0F0F0Fu) | ((Q[i] >> 2) & 0x30303030u);
        p0 = dp2a_lo(X.v[2 * i], v0, p0);
        p0 = dp2a_hi(X.v[2 * i + 1], v0, p0);
        p1 = dp2a_lo(X.v[8 + 2 * i], v1, p1);
        p1 = dp2a_hi(X.v[8 + 2 * i + 1], v1, p1);
        p2 = dp2a_lo(X.v[16 + 2 * i], v2, p2);
        p2 = dp2a_hi(X.v[16 + 2 * i + 1], v2, p2);
        p3 = dp2a_lo(X.v[24 + 2 * i], v3, p3);
        p3 = dp2a_hi(X.v[24 + 2 * i + 1], v3, p3);
    }
    const uint32_t *sq = reinterpret_cast<const uint32_t *>(blk + 192 + 8 * h - L.sh);
    const uint32_t w0 = sq[0], w1 = sq[1], w2 = sq[2];
    const uint32_t slo = prmt(w0, w1, L.sel), shi = prmt(w1, w2, L.sel);
    const int sc0 = (int)prmt(slo, 0u, L.ssel[0]);
    const int sc1 = (int)prmt(slo, 0u, L.ssel[1]);
    const int sc2 = (int)prmt(shi, 0u, L.ssel[0]);
    const int sc3 = (int)prmt(shi, 0u, L.ssel[1]);
    float acc = (s2f_small(sc0) * X.s[0]) * (float)(p0 - X.c[0]);
    acc = fmaf(s2f_small(sc1) * X.s[1], (float)(p1 - X.c[1]), acc);
    acc = fmaf(s2f_small(sc2) * X.s[2], (float)(p2 - X.c[2]), acc);
    acc = fmaf(s2f_small(sc3) * X.s[3], (float)(p3 - X.c[3]), acc);
    const float d = __half2float(*reinterpret_cast<const __half *>(blk + 208));
    return d * acc;
}

// ---------------------------------------------------------------------------
// weights-stationary lane dots: a lane decodes its share of a block row once
// and applies it to several tokens.  The activation side is the same int16
// slice (xq_pos layout) with its group scales xs (per 32 values) and exact
// int sums xs16 (per 16 values) computed when the activations were quantised.
// ---------------------------------------------------------------------------
// Q4_K lane (block b, pair g): the 32 quant bytes of sub-blocks 2g, 2g+1 and
// their factors d*sc (the high-nibble one carrying 1/16) and dmin*m.
struct Q4W {
    uint32_t w[8];
    float a0, a1, b0, b1;
};
__device__ __forceinline__ void q4k_lane_w(Q4W &W, const uint8_t *blk, int g)
{
    const uint4 hd = *reinterpret_cast<const uint4 *>(blk);
    const uint4 qa = *reinterpret_cast<const uint4 *>(blk + 16 + 32 * g);
    const uint4 qb = *reinterpret_cast<const uint4 *>(blk + 32 + 32 * g);
    W.w[0] = qa.x;
    W.w[1] = qa.y;
    W.w[2] = qa.z;
    W.w[3] = qa.w;
    W.w[4] = qb.x;
    W.w[5] = qb.y;
    W.w[6] = qb.z;
    W.w[7] = qb.w;
    const uint32_t sh = 16u * (uint32_t)(g & 1);
    const uint32_t A = hd.y >> sh, B = hd.z >> sh, C = hd.w >> sh;
    uint32_t scp, mp;
    if (g >= 2) {
        scp = (C & 0x0F0Fu) | ((A >> 2) & 0x3030u);
        mp = ((C >> 4) & 0x0F0Fu) | ((B >> 2) & 0x3030u);
    } else {
        scp = A & 0x3F3Fu;
        mp = B & 0x3F3Fu;
    }
    const float2 dd = __half22float2(*reinterpret_cast<const __half2 *>(&hd.x));
    W.a0 = dd.x * u2f_small(scp & 0xFFu);
    W.a1 = dd.x * (u2f_small((scp >> 8) & 0xFFu) * 0.0625f);
    W.b0 = dd.y * u2f_small(mp & 0xFFu);
    W.b1 = dd.y * u2f_small((mp >> 8) & 0xFFu);
}
// One token's dot with a decoded Q4_K lane; e0 = 256*b + 64*g, rs scales xs.
__device__ __forceinline__ float q4k_dot_w(const Q4W &W, const int16_t *xq, const float *xs, const int *xs16, int e0,
                                           float rs)
{
    int p0 = 0, p1 = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int4 t = xq_piece(xq, e0 + 8 * k);
        const uint32_t l0 = W.w[2 * k] & 0x0F0F0F0Fu, l1 = W.w[2 * k + 1] & 0x0F0F0F0Fu;
        p0 = dp2a_lo(t.x, l0, p0);
        p0 = dp2a_hi(t.y, l0, p0);
        p0 = dp2a_lo(t.z, l1, p0);
        p0 = dp2a_hi(t.w, l1, p0);
        const int4 u = xq_piece(xq, e0 + 32 + 8 * k);
        const uint32_t h0 = W.w[2 * k] & 0xF0F0F0F0u, h1 = W.w[2 * k + 1] & 0xF0F0F0F0u;
        p1 = dp2a_lo(u.x, h0, p1);
        p1 = dp2a_hi(u.y, h0, p1);
        p1 = dp2a_lo(u.z, h1, p1);
        p1 = dp2a_hi(u.w, h1, p1);
    }
    const int gi = e0 >> 5;
    const float f0 = xs[gi] * rs, f1 = xs[gi + 1] * rs;
    const int s0 = xs16[2 * gi] + xs16[2 * gi + 1], s1 = xs16[2 * gi + 2] + xs16[2 * gi + 3];
    const float mins = fmaf(W.b1 * f1, (float)s1, (W.b0 * f0) * (float)s0);
    return fmaf(W.a0 * f0, (float)p0, fmaf(W.a1 * f1, (float)p1, -mins));
}

// Q6_K lane (half h, l-group g): the 6-bit codes of its four runs and d*sc.
struct Q6W {
    uint32_t v[16];  // v[4r + i]: codes of run r, l = 16g + 4i .. 4i + 3
    float s[4];
};
__device__ __forceinline__ void q6k_lane_w(Q6W &W, const uint8_t *blk, int h, int g, const Q6Lane &L)
{
    uint32_t A[4], B[4], Q[4];
    ld16_shift(blk + 64 * h + 16 * g, L.sh, L.sel, A);
    ld16_shift(blk + 64 * h + 32 + 16 * g, L.sh, L.sel, B);
    ld16_shift(blk + 128 + 32 * h + 16 * g, L.sh, L.sel, Q);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        W.v[i] = (A[i] & 0x0F0F0F0Fu) | ((Q[i] << 4) & 0x30303030u);
        W.v[4 + i] = (B[i] & 0x0F0F0F0Fu) | ((Q[i] << 2) & 0x30303030u);
        W.v[8 + i] = ((A[i] >> 4) & 0x0F0F0F0Fu) | (Q[i] & 0x30303030u);
        W.v[12 + i] = ((B[i] >> 4) & 0x0F0F0F0Fu) | ((Q[i] >> 2) & 0x30303030u);
    }
    const uint32_t *sq = reinterpret_cast<const uint32_t *>(blk + 192 + 8 * h - L.sh);
    const uint32_t w0 = sq[0], w1 = sq[1], w2 = sq[2];
    const uint32_t slo = prmt(w0, w1, L.sel), shi = prmt(w1, w2, L.sel);
    const float d = __half2float(*reinterpret_cast<const __half *>(blk + 208));
    W.s[0] = d * s2f_small((int)prmt(slo, 0u, L.ssel[0]));
    W.s[1] = d * s2f_small((int)prmt(slo, 0u, L.ssel[1]));
    W.s[2] = d * s2f_small((int)prmt(shi, 0u, L.ssel[0]));
    W.s[3] = d * s2f_small((int)prmt(shi, 0u, L.ssel[1]));
}
// One token's dot with a decoded Q6_K lane; base = 256*b + 128*h.
__device__ __forceinline__ float q6k_dot_w(const Q6W &W, const int16_t *xq, const float *xs, const int *xs16, int base,
                                           int g, float rs)
{
    float acc = 0.0f;
#pragma unroll
    for (int r = 0; r < 4; ++r) {
        const int e = base + 32 * r + 16 * g;
        const int4 t0 = xq_piece(xq, e), t1 = xq_piece(xq, e + 8);
        int p = dp2a_lo(t0.x, W.v[4 * r], 0);
        p = dp2a_hi(t0.y, W.v[4 * r], p);
        p = dp2a_lo(t0.z, W.v[4 * r + 1], p);
        p = dp2a_hi(t0.w, W.v[4 * r + 1], p);
        p = dp2a_lo(t1.x, W.v[4 * r + 2], p);
        p = dp2a_hi(t1.y, W.v[4 * r + 2], p);
        p = dp2a_lo(t1.z, W.v[4 * r + 3], p);
        p = dp2a_hi(t1.w, W.v[4 * r + 3], p);
        acc = fmaf(W.s[r] * (xs[e >> 5] * rs), (float)(p - 32 * xs16[e >> 4]), acc);
    }
    return acc;
}

// Exact int sums of a quantised group's two 16-value halves (full warp, one
// value per lane): lanes 0 and 16 return their half's sum.
__device__ __forceinline__ int sum16(int q)
{
#pragma unroll
    for (int o = 8; o; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
    return q;
}

}  // namespace bread
