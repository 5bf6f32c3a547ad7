// ws3d_lean.cuh -- the default-face cell rule with fewer instructions.
//
// Same results, bit for bit, as cell_rule<false> / cells4_default (the
// reference order of separately rounded f32 operations), computed with
//  * packed f32x2 add / sub / mul (sm_100): two IEEE round-to-nearest f32
//    operations per instruction, each rounding exactly like __fadd_rn etc.
//    The code generator may contract a packed multiply that feeds a packed
//    add into a fused multiply-add even with .rn (measured: 1-ulp
//    differences), so no inexact packed product feeds an add here: 2c and 4c
//    are exact doublings and 6c = round(4c + 2c) = round(6 * c); c2 * lap is
//    two scalar __fmul_rn, which are never contracted;
//  * a branch-free sponge: the sponge table F(d) (d < width) is
//    non-decreasing with F <= 1, and F(d) = 1 for d >= width, so
//    F(min(dx, dy, dz)) = min(F(min(dx, dy)), F(dz)); the row factor is
//    precomputed per lane, the plane factor per plane, and cells outside the
//    sponge are multiplied by exactly 1.0f (v * 1.0f == v);
//  * interior / boundary chosen by a select instead of branches.
// Difference in cells nobody reads: pitch padding columns (x >= W) get
// p_prev * 0.1 instead of p_prev; they are never an interior cell's
// neighbour and never leave the device.
// The host enables these kernels only when the sponge table is monotone.
#pragma once

#include "ws3d_kernels.cuh"

namespace ws3d {

typedef unsigned long long f2;  // two f32 in one 64-bit register pair (lo = first)

__device__ __forceinline__ f2 pk(float lo, float hi) {
    f2 r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ void upk(f2 v, float& lo, float& hi) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ f2 add2(f2 a, f2 b) {
    f2 r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ f2 sub2(f2 a, f2 b) {
    f2 r;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ f2 mul2(f2 a, f2 b) {
    f2 r;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}

struct LeanConst {
    f2 damp, refl;
};
__device__ __forceinline__ LeanConst lean_const(float damping) {
    return LeanConst{pk(damping, damping), pk(kFaceReflection, kFaceReflection)};
}

// Sponge factor of face distance d (1.0f outside the sponge).
__device__ __forceinline__ float sponge_f(uint32_t d, const StepParams& a) {
    return d < a.sponge_w ? __ldg(a.sponge + d) : 1.0f;
}

// Per lane and row: interior bits of cells x..x+3 (in x and y) and their
// sponge factors F(min(dx, dy)) (1.0f for boundary cells).  x and y may have
// wrapped below zero (halo rows / columns of a tile at the grid edge): those
// cells are not interior.
struct LeanRow {
    float fx[4];
    uint32_t bits;
};
__device__ __forceinline__ bool lean_in(uint32_t v, uint32_t n) { return v >= 1 && v + 1 < n && v < n; }

__device__ __forceinline__ LeanRow make_lean_row(uint32_t x, uint32_t y, const StepParams& a) {
    LeanRow r;
    r.bits = 0;
    const bool yin = lean_in(y, a.H);
    const uint32_t dy = yin ? min(y, a.H - 1 - y) : 0u;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const uint32_t xk = x + k;
        const bool in = yin && lean_in(xk, a.W);
        if (in) r.bits |= 1u << k;
        r.fx[k] = in ? sponge_f(min(min(xk, a.W - 1 - xk), dy), a) : 1.0f;
    }
    return r;
}

// Plane terms: interior mask of the row's cells at global plane zg and the
// plane's sponge factor.
__device__ __forceinline__ uint32_t lean_mask(uint32_t bits, uint32_t zg, const StepParams& a) {
    return (zg >= 1 && zg + 1 < a.Dg) ? bits : 0u;
}
__device__ __forceinline__ float lean_fz(uint32_t zg, const StepParams& a) {
    return (zg < a.Dg) ? sponge_f(min(zg, a.Dg - 1 - zg), a) : 1.0f;
}

// Four cells of a row.  m: interior mask (bit k = cell x+k), fx: row sponge
// factors, fz: plane sponge factor; wl / er: the x neighbours left of x and
// right of x+3; S/N: y-1 / y+1; D/U: z-1 / z+1; C: the cells; PV: p_prev.
__device__ __forceinline__ float4 cells4_lean(uint32_t m, const float (&fx)[4], float fz, float wl,
                                              float er, float4 S, float4 N, float4 D, float4 C,
                                              float4 U, float4 PV, float4 C2, const LeanConst& k) {
    const f2 c01 = pk(C.x, C.y), c23 = pk(C.z, C.w);
    const f2 w01 = pk(wl, C.x), w23 = pk(C.y, C.z);  // west neighbours
    const f2 e23 = pk(C.w, er);                      // east of cells 2, 3; east of 0, 1 = w23
    f2 t01 = add2(w01, w23), t23 = add2(w23, e23);
    t01 = add2(t01, pk(S.x, S.y));
    t23 = add2(t23, pk(S.z, S.w));
    t01 = add2(t01, pk(N.x, N.y));
    t23 = add2(t23, pk(N.z, N.w));
    t01 = add2(t01, pk(D.x, D.y));
    t23 = add2(t23, pk(D.z, D.w));
    t01 = add2(t01, pk(U.x, U.y));
    t23 = add2(t23, pk(U.z, U.w));
    const f2 d01 = add2(c01, c01), d23 = add2(c23, c23);  // 2c (exact)
    t01 = sub2(t01, add2(add2(d01, d01), d01));             // lap - 6c, 6c = round(4c + 2c)
    t23 = sub2(t23, add2(add2(d23, d23), d23));
    float l0, l1, l2, l3;
    upk(t01, l0, l1);
    upk(t23, l2, l3);
    const f2 pv01 = pk(PV.x, PV.y), pv23 = pk(PV.z, PV.w);
    f2 n01 = add2(sub2(d01, pv01), pk(__fmul_rn(C2.x, l0), __fmul_rn(C2.y, l1)));
    f2 n23 = add2(sub2(d23, pv23), pk(__fmul_rn(C2.z, l2), __fmul_rn(C2.w, l3)));
    n01 = mul2(n01, k.damp);
    n23 = mul2(n23, k.damp);
    n01 = mul2(n01, pk(fminf(fx[0], fz), fminf(fx[1], fz)));
    n23 = mul2(n23, pk(fminf(fx[2], fz), fminf(fx[3], fz)));
    const f2 r01 = mul2(pv01, k.refl), r23 = mul2(pv23, k.refl);
    float a0, a1, a2, a3, b0, b1, b2, b3;
    upk(n01, a0, a1);
    upk(n23, a2, a3);
    upk(r01, b0, b1);
    upk(r23, b2, b3);
    return make_float4((m & 1u) ? a0 : b0, (m & 2u) ? a1 : b1, (m & 4u) ? a2 : b2,
                       (m & 8u) ? a3 : b3);
}

// Interior update of four cells, without sponge and boundary handling (the
// caller fixes up the lanes that have sponge or boundary cells, see
// cells4_fixup): per cell ((((w+e)+s)+n)+d)+u, - 6c, (2c - p_prev) + c2 * lap,
// * damping.  w + e and the products 6c and c2 * lap are scalar (the shifted
// w / e pairs would need register moves; scalar products are never
// contracted); 2c is an exact doubling.
__device__ __forceinline__ float4 cells4_fast(float wl, float er, float4 S, float4 N, float4 D,
                                              float4 C, float4 U, float4 PV, float4 C2, f2 damp) {
    f2 t01 = pk(__fadd_rn(wl, C.y), __fadd_rn(C.x, C.z));
    f2 t23 = pk(__fadd_rn(C.y, C.w), __fadd_rn(C.z, er));
    t01 = add2(t01, pk(S.x, S.y));
    t23 = add2(t23, pk(S.z, S.w));
    t01 = add2(t01, pk(N.x, N.y));
    t23 = add2(t23, pk(N.z, N.w));
    t01 = add2(t01, pk(D.x, D.y));
    t23 = add2(t23, pk(D.z, D.w));
    t01 = add2(t01, pk(U.x, U.y));
    t23 = add2(t23, pk(U.z, U.w));
    t01 = sub2(t01, pk(__fmul_rn(6.0f, C.x), __fmul_rn(6.0f, C.y)));
    t23 = sub2(t23, pk(__fmul_rn(6.0f, C.z), __fmul_rn(6.0f, C.w)));
    const f2 c01 = pk(C.x, C.y), c23 = pk(C.z, C.w);
    const f2 b01 = sub2(add2(c01, c01), pk(PV.x, PV.y));
    const f2 b23 = sub2(add2(c23, c23), pk(PV.z, PV.w));
    float l0, l1, l2, l3;
    upk(t01, l0, l1);
    upk(t23, l2, l3);
    f2 n01 = add2(b01, pk(__fmul_rn(C2.x, l0), __fmul_rn(C2.y, l1)));
    f2 n23 = add2(b23, pk(__fmul_rn(C2.z, l2), __fmul_rn(C2.w, l3)));
    n01 = mul2(n01, damp);
    n23 = mul2(n23, damp);
    float4 o;
    upk(n01, o.x, o.y);
    upk(n23, o.z, o.w);
    return o;
}

// Sponge and boundary for the lanes that need them: interior cells in the
// sponge are multiplied by F(d) = min(fx_k, fz) (v * 1.0f == v elsewhere),
// cells that are not interior (mask bit clear) become p_prev * 0.1.
__device__ __forceinline__ float4 cells4_fixup(float4 v, bool sponge, const float (&fx)[4], float fz,
                                               uint32_t m, float4 PV) {
    if (sponge) {
        v.x = __fmul_rn(v.x, fminf(fx[0], fz));
        v.y = __fmul_rn(v.y, fminf(fx[1], fz));
        v.z = __fmul_rn(v.z, fminf(fx[2], fz));
        v.w = __fmul_rn(v.w, fminf(fx[3], fz));
    }
    if (m != 0xFu) {
        if (!(m & 1u)) v.x = __fmul_rn(PV.x, kFaceReflection);
        if (!(m & 2u)) v.y = __fmul_rn(PV.y, kFaceReflection);
        if (!(m & 4u)) v.z = __fmul_rn(PV.z, kFaceReflection);
        if (!(m & 8u)) v.w = __fmul_rn(PV.w, kFaceReflection);
    }
    return v;
}

// Branch-free sponge: v_k *= min(fx_k, fz) for all four cells (a factor of
// exactly 1.0f outside the sponge leaves v unchanged), then cells that are
// not interior (mask bit clear) become p_prev * 0.1.
__device__ __forceinline__ float4 cells4_finish(float4 v, const float (&fx)[4], float fz,
                                               uint32_t m, float4 PV) {
    f2 lo = mul2(pk(v.x, v.y), pk(fminf(fx[0], fz), fminf(fx[1], fz)));
    f2 hi = mul2(pk(v.z, v.w), pk(fminf(fx[2], fz), fminf(fx[3], fz)));
    upk(lo, v.x, v.y);
    upk(hi, v.z, v.w);
    if (m != 0xFu) v = cells4_fixup(v, false, fx, fz, m, PV);
    return v;
}

// One cell (scalar), same rule.
__device__ __forceinline__ float cell1_lean(bool interior, float f, float w, float e, float s,
                                            float n, float dn, float up, float c, float pv, float c2,
                                            float damping) {
    float lap = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(w, e), s), n), dn), up);
    lap = __fsub_rn(lap, __fmul_rn(6.0f, c));
    float v = __fadd_rn(__fsub_rn(__fmul_rn(2.0f, c), pv), __fmul_rn(c2, lap));
    v = __fmul_rn(__fmul_rn(v, damping), f);
    return interior ? v : __fmul_rn(pv, kFaceReflection);
}

}  // namespace ws3d
