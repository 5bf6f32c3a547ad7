// ws3d_kernels.cuh -- sm_100a device code for the WaveSim3D FDTD step.
//
// Device layout (HBM): every field is stored pitched.  A row holds `pitch`
// floats (W rounded up to a multiple of 32, so every row starts on a
// 128-byte boundary); a plane holds H rows; a slab holds the owned planes
// plus one ghost plane below and one above.  Kernel pointers address owned
// plane 0, so plane index -1 and nz are the ghosts.  Padding columns
// (x >= W) are kept at zero: the kernels write them back unchanged.
//
// Arithmetic: every multiply and add is an explicitly rounded intrinsic
// (__fadd_rn / __fmul_rn ...), which the compiler never contracts into an
// FMA, in the operation order of the reference CPU step
// (crates/ringkernel-wavesim3d/src/simulation/grid3d.rs:238-256).  Results
// are therefore bit-identical to the reference arithmetic.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include "ws3d_index.h"

namespace ws3d {

constexpr uint8_t kNormal = 0, kAbsorber = 1, kReflector = 2, kObstacle = 3;
constexpr float kFaceReflection = 0.1f;  // grid3d.rs:111

struct StepParams {
    const float* p;         // pressure (read), owned plane 0
    float* pp;              // pressure_prev (read, then overwritten with the new field)
    const float* c2f;       // per-cell Courant^2 or nullptr
    const uint8_t* types;   // per-cell CellType or nullptr (default face layout)
    const float* refl;      // per-cell reflection (with types)
    const float* sponge;    // sponge table s[d], d < sponge_w
    uint32_t W, H, pitch;   // global width/height, row pitch (floats)
    uint32_t nz;            // owned planes
    uint32_t z0;            // global z of owned plane 0
    uint32_t Dg;            // global depth
    uint64_t plane;         // H * pitch
    float c2, damping;
    uint32_t sponge_w;
    // z-slab halo exchange (all null / zero on a single GPU)
    float* peer_lo;                      // lower neighbour's upper ghost plane (new field)
    float* peer_hi;                      // upper neighbour's lower ghost plane (new field)
    float* peer_lo2;                     // temporal depth 2: its second upper ghost plane, or null
    float* peer_hi2;                     // temporal depth 2: its second lower ghost plane, or null
    const unsigned long long* wait_lo;   // flag the lower neighbour raises, or null
    const unsigned long long* wait_hi;   // flag the upper neighbour raises, or null
    unsigned long long wait_val;         // both flags must reach this value first
    unsigned long long budget_ns;        // bounded wait
    unsigned int* status;                // error word (bit 0: lower wait, bit 1: upper wait)
    // [0] device ns spent in neighbour-flag waits that did not pass at once,
    // [1] the number of such waits (both summed over launches; z-slabs)
    unsigned long long* wait_acc;
};

// ---------------------------------------------------------------------------
// System-scope flag protocol for the z-slab exchange.  Every wait is bounded
// by a %globaltimer budget and a hard iteration cap; when it gives up it
// records the failure in the status word and returns, so a missing neighbour
// never hangs the GPU.
// ---------------------------------------------------------------------------
__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys(unsigned long long* p, unsigned long long v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// `acc` (optional): a wait that did not pass at once adds its duration in ns
// to acc[0] and 1 to acc[1].
__device__ __noinline__ bool wait_flag_geq(const unsigned long long* f, unsigned long long v,
                                           unsigned long long budget_ns,
                                           unsigned long long* acc = nullptr) {
    if (ld_acquire_sys(f) >= v) return true;
    const unsigned long long t0 = global_ns();
    bool ok = false;
    for (unsigned int it = 1; it < (1u << 26); ++it) {
        __nanosleep(128);
        if (ld_acquire_sys(f) >= v) {
            ok = true;
            break;
        }
        if ((it & 31u) == 0 && global_ns() - t0 > budget_ns) break;
    }
    if (acc) {
        atomicAdd(acc, global_ns() - t0);
        atomicAdd(acc + 1, 1ull);
    }
    return ok;
}

// Raise the neighbours' flags after this GPU's step kernel has completed
// (stream order) and its peer stores were fenced at system scope.
__global__ void k_halo_signal(unsigned long long* flag_lo, unsigned long long* flag_hi,
                              unsigned long long v) {
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    __threadfence_system();
    if (flag_lo) st_release_sys(flag_lo, v);
    if (flag_hi) st_release_sys(flag_hi, v);
}

__device__ __forceinline__ float4 ld4(const float* p) {
    return __ldg(reinterpret_cast<const float4*>(p));
}
// Streamed once per step: keep it out of L1, normal L2 policy.
__device__ __forceinline__ float4 ld4_stream(const float* p) {
    return __ldcs(reinterpret_cast<const float4*>(p));
}
__device__ __forceinline__ void st4(float* p, float4 v) {
    *reinterpret_cast<float4*>(p) = v;
}
// Ghost planes may be written by a peer GPU while this kernel runs (after
// the flag wait): read them through L2 (coherent), never the non-coherent path.
__device__ __forceinline__ float4 ld4_plane(const float* p, int64_t z, uint32_t nz) {
    if (z < 0 || z >= (int64_t)nz) return __ldcg(reinterpret_cast<const float4*>(p));
    return __ldg(reinterpret_cast<const float4*>(p));
}

// Reference update of one interior Normal cell (grid3d.rs:250-256), then the
// optional sponge multiply.
__device__ __forceinline__ float leapfrog(float w, float e, float s, float n, float dn,
                                          float up, float c, float pprev, float c2,
                                          float damping) {
    float lap = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(w, e), s), n), dn), up);
    lap = __fsub_rn(lap, __fmul_rn(6.0f, c));
    float pn = __fadd_rn(__fsub_rn(__fmul_rn(2.0f, c), pprev), __fmul_rn(c2, lap));
    return __fmul_rn(pn, damping);
}

__device__ __forceinline__ uint32_t face_dist(uint32_t x, uint32_t y, uint32_t zg,
                                              const StepParams& a) {
    uint32_t d = min(x, a.W - 1 - x);
    d = min(d, min(y, a.H - 1 - y));
    d = min(d, min(zg, a.Dg - 1 - zg));
    return d;
}

// Full cell rule: stencil for interior Normal cells, keep p_prev otherwise,
// then the boundary multiply for Absorber/Obstacle (grid3d.rs:353-370).
template <bool kCells>
__device__ __forceinline__ float cell_rule(uint32_t x, uint32_t y, uint32_t zg, bool interior,
                                           float w, float e, float s, float n, float dn,
                                           float up, float c, float pprev, float c2,
                                           uint8_t t, float r, const StepParams& a) {
    float v = pprev;
    bool normal = kCells ? (t == kNormal) : interior;
    if (interior && normal) {
        v = leapfrog(w, e, s, n, dn, up, c, pprev, c2, a.damping);
        if (a.sponge_w) {
            uint32_t d = face_dist(x, y, zg, a);
            if (d < a.sponge_w) v = __fmul_rn(v, __ldg(a.sponge + d));
        }
    }
    if (kCells) {
        if (t == kAbsorber || t == kObstacle) v = __fmul_rn(v, r);
    } else {
        if (!interior && x < a.W) v = __fmul_rn(v, kFaceReflection);
    }
    return v;
}

// x/y part of the default-face cell rule for one thread's float4 column,
// computed once per (tile) run: which of the 4 cells are interior in x and y,
// which are real cells (x < W, not row padding), and min(dx, dy) for the
// sponge.  Per plane only the z part is added (cells4_default).
struct XYPre {
    uint32_t dxy01, dxy23;  // min(dx, dy) of cells 0..3, 16 bits each (clamped to 65535)
    uint32_t bits;          // bit k: cell x+k interior in x and y; bit 4+k: x+k < W
};

__device__ __forceinline__ XYPre make_xypre(uint32_t x, uint32_t y, const StepParams& a) {
    XYPre q;
    q.bits = 0;
    const bool yin = y >= 1 && y + 1 < a.H;
    const uint32_t dy = min(y, a.H - 1 - y);
    uint32_t d[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const uint32_t xk = x + k;
        const bool xin = xk >= 1 && xk + 1 < a.W;
        if (xin && yin) q.bits |= 1u << k;
        if (xk < a.W) q.bits |= 16u << k;
        d[k] = (xin && yin) ? min(min(min(xk, a.W - 1 - xk), dy), 65535u) : 0u;
    }
    q.dxy01 = d[0] | (d[1] << 16);
    q.dxy23 = d[2] | (d[3] << 16);
    return q;
}

__device__ __forceinline__ uint32_t xypre_dxy(const XYPre& q, int k) {
    const uint32_t w = k < 2 ? q.dxy01 : q.dxy23;
    return (k & 1) ? (w >> 16) : (w & 0xFFFFu);
}

// The default-face cell rule for 4 cells at global plane zg; bit-identical to
// cell_rule<false> (same operations in the same order).
__device__ __forceinline__ float4 cells4_default(const XYPre& q, uint32_t zg, float wl, float er,
                                                 float4 S, float4 N, float4 pm, float4 pc,
                                                 float4 pn, float4 vpp, float4 c2,
                                                 const StepParams& a) {
    const bool zin = zg >= 1 && zg + 1 < a.Dg;
    const uint32_t dz = min(zg, a.Dg - 1 - zg);
    const float w[4] = {wl, pc.x, pc.y, pc.z};
    const float e[4] = {pc.y, pc.z, pc.w, er};
    const float s[4] = {S.x, S.y, S.z, S.w};
    const float n[4] = {N.x, N.y, N.z, N.w};
    const float d[4] = {pm.x, pm.y, pm.z, pm.w};
    const float u[4] = {pn.x, pn.y, pn.z, pn.w};
    const float c[4] = {pc.x, pc.y, pc.z, pc.w};
    const float pv[4] = {vpp.x, vpp.y, vpp.z, vpp.w};
    const float cc[4] = {c2.x, c2.y, c2.z, c2.w};
    float o[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        float v = pv[k];
        if (zin && ((q.bits >> k) & 1u)) {
            v = leapfrog(w[k], e[k], s[k], n[k], d[k], u[k], c[k], pv[k], cc[k], a.damping);
            if (a.sponge_w) {
                // dxy is clamped to 65535 >= any sponge width (<= 4096): same test
                const uint32_t dist = min(xypre_dxy(q, k), dz);
                if (dist < a.sponge_w) v = __fmul_rn(v, __ldg(a.sponge + dist));
            }
        } else if ((q.bits >> (4 + k)) & 1u) {
            v = __fmul_rn(v, kFaceReflection);
        }
        o[k] = v;
    }
    return make_float4(o[0], o[1], o[2], o[3]);
}

__device__ __forceinline__ bool is_interior(uint32_t x, uint32_t y, uint32_t zg,
                                            const StepParams& a) {
    return x >= 1 && x + 1 < a.W && y >= 1 && y + 1 < a.H && zg >= 1 && zg + 1 < a.Dg;
}

// ---------------------------------------------------------------------------
// Z-streaming step kernel.
//
// CTA = 32 x TY threads covering a 128 x TY tile of an xy plane; the CTA walks
// its tile through z planes [zb, ze).  Each thread owns one float4 column
// (4 consecutive x).  Per plane it reads p (the front plane z+1), p_prev and
// optionally c2 with 128-bit loads and writes the new field with one 128-bit
// store: 12 (16 with c2) bytes per cell from HBM.  z neighbours come from a
// three-plane register queue, x neighbours from the float4 itself plus warp
// shuffles (one halo float at each end of the warp), y neighbours from the
// current plane staged in shared memory with one halo row above and below.
// Loads for plane z+1 are issued one iteration ahead.
// ---------------------------------------------------------------------------
// One CTA (32 x TY threads) computes planes [zb, ze) of tile (bx, by).  Its
// staging arrays are declared __shared__ here (one set per instantiation, so
// the compiler addresses them as shared memory).  Ends with a CTA barrier so
// it can be called again by a persistent loop.
template <bool kC2F, bool kCells, int TY>
__device__ __forceinline__ void zs_tile(const StepParams& a, uint32_t bx, uint32_t by,
                                        uint32_t zb, uint32_t ze) {
    static_assert(TY >= 2, "the y-halo rows need two distinct warps");
    __shared__ float4 srow[2][TY + 2][32];
    __shared__ float shl[2][TY], shr[2][TY];
    const int lane = threadIdx.x, w = threadIdx.y;
    const bool halo_wait = a.wait_lo != nullptr || a.wait_hi != nullptr;

    // Boundary chunks read ghost planes that a neighbour GPU writes: wait
    // (bounded) for its flag.  Interior chunks never wait and are scheduled
    // first, so they overlap the exchange.
    if (halo_wait) {
        const bool need_lo = a.wait_lo && zb == 0;
        const bool need_hi = a.wait_hi && ze == a.nz;
        if (need_lo || need_hi) {
            if (threadIdx.x == 0 && threadIdx.y == 0) {
                unsigned int bad = 0;
                if (need_lo && !wait_flag_geq(a.wait_lo, a.wait_val, a.budget_ns, a.wait_acc)) bad |= 1u;
                if (need_hi && !wait_flag_geq(a.wait_hi, a.wait_val, a.budget_ns, a.wait_acc)) bad |= 2u;
                if (bad) atomicOr(a.status, bad);
            }
            __syncthreads();
        }
    }
    const ZsLane L = zs_lane<TY>(bx, by, lane, w, a.W, a.H, a.pitch);
    const bool act = L.act, ylo = L.ylo, yhi = L.yhi, xl = L.xl, xr = L.xr;
    const uint32_t x = L.x, y = L.y;
    XYPre xy{};
    if (!kCells) xy = make_xypre(x, y, a);
    const int64_t P = (int64_t)a.plane;
    const int64_t row = L.row;

    const float4 z4 = make_float4(0.f, 0.f, 0.f, 0.f);
    const float* __restrict__ p = a.p;
    float* __restrict__ pp = a.pp;

    // Prologue: planes zb-1, zb in registers; plane zb staged in smem.
    const int64_t ozb = zs_plane((int64_t)zb, P);
    float4 pm = act ? ld4_plane(p + zs_plane((int64_t)zb - 1, P) + row, (int64_t)zb - 1, a.nz) : z4;
    float4 pc = act ? ld4(p + ozb + row) : z4;
    srow[0][w + 1][lane] = pc;
    if (ylo) srow[0][0][lane] = ld4(p + ozb + L.rowlo);
    if (yhi) srow[0][TY + 1][lane] = ld4(p + ozb + L.rowhi);
    if (xl) shl[0][w] = __ldg(p + ozb + L.offxl);
    if (xr) shr[0][w] = __ldg(p + ozb + L.offxr);
    float4 pn = act ? ld4_plane(p + zs_plane((int64_t)zb + 1, P) + row, (int64_t)zb + 1, a.nz) : z4;
    float4 vpp = act ? ld4_stream(pp + ozb + row) : z4;
    float4 vc2 = (kC2F && act) ? ld4_stream(a.c2f + ozb + row) : z4;
    uchar4 vt = make_uchar4(0, 0, 0, 0);
    if (kCells && act) vt = *reinterpret_cast<const uchar4*>(a.types + ozb + row);
    __syncthreads();

    int cur = 0;
    for (uint32_t zl = zb; zl < ze; ++zl) {
        const bool more = zl + 1 < ze;
        // Prefetch for plane zl+1 (and the front plane zl+2).
        float4 pn2 = z4, vpp2 = z4, vc22 = z4, hy = z4;
        float hx = 0.f;
        uchar4 vt2 = make_uchar4(0, 0, 0, 0);
        if (more) {
            const int64_t zo1 = zs_plane((int64_t)zl + 1, P);
            if (act) {
                pn2 = ld4_plane(p + zs_plane((int64_t)zl + 2, P) + row, (int64_t)zl + 2, a.nz);
                vpp2 = ld4_stream(pp + zo1 + row);
                if (kC2F) vc22 = ld4_stream(a.c2f + zo1 + row);
                if (kCells) vt2 = *reinterpret_cast<const uchar4*>(a.types + zo1 + row);
            }
            if (ylo) hy = ld4(p + zo1 + L.rowlo);
            else if (yhi) hy = ld4(p + zo1 + L.rowhi);
            if (xl) hx = __ldg(p + zo1 + L.offxl);
            else if (xr) hx = __ldg(p + zo1 + L.offxr);
        }

        // Compute plane zl.
        const float4 S = srow[cur][w][lane];
        const float4 N = srow[cur][w + 2][lane];
        float wl = __shfl_up_sync(0xffffffffu, pc.w, 1);
        float er = __shfl_down_sync(0xffffffffu, pc.x, 1);
        if (lane == 0) wl = shl[cur][w];
        if (lane == 31) er = shr[cur][w];

        if (act && !kCells) {
            const int64_t o = zs_plane((int64_t)zl, P) + row;
            const float4 c2v = kC2F ? vc2 : make_float4(a.c2, a.c2, a.c2, a.c2);
            const float4 out = cells4_default(xy, a.z0 + zl, wl, er, S, N, pm, pc, pn, vpp, c2v, a);
            st4(pp + o, out);
            if (zl == 0 && a.peer_lo) st4(a.peer_lo + row, out);
            if (zl + 1 == a.nz && a.peer_hi) st4(a.peer_hi + row, out);
        } else if (act) {
            const uint32_t zg = a.z0 + zl;
            const int64_t o = zs_plane((int64_t)zl, P) + row;
            float4 out;
            float c2x = kC2F ? vc2.x : a.c2, c2y = kC2F ? vc2.y : a.c2;
            float c2z = kC2F ? vc2.z : a.c2, c2w = kC2F ? vc2.w : a.c2;
            float r0 = 0.f, r1 = 0.f, r2 = 0.f, r3 = 0.f;
            if (kCells) {
                if (vt.x == kAbsorber || vt.x == kObstacle) r0 = __ldg(a.refl + o + 0);
                if (vt.y == kAbsorber || vt.y == kObstacle) r1 = __ldg(a.refl + o + 1);
                if (vt.z == kAbsorber || vt.z == kObstacle) r2 = __ldg(a.refl + o + 2);
                if (vt.w == kAbsorber || vt.w == kObstacle) r3 = __ldg(a.refl + o + 3);
            }
            out.x = cell_rule<kCells>(x + 0, y, zg, is_interior(x + 0, y, zg, a), wl, pc.y, S.x,
                                      N.x, pm.x, pn.x, pc.x, vpp.x, c2x, vt.x, r0, a);
            out.y = cell_rule<kCells>(x + 1, y, zg, is_interior(x + 1, y, zg, a), pc.x, pc.z,
                                      S.y, N.y, pm.y, pn.y, pc.y, vpp.y, c2y, vt.y, r1, a);
            out.z = cell_rule<kCells>(x + 2, y, zg, is_interior(x + 2, y, zg, a), pc.y, pc.w,
                                      S.z, N.z, pm.z, pn.z, pc.z, vpp.z, c2z, vt.z, r2, a);
            out.w = cell_rule<kCells>(x + 3, y, zg, is_interior(x + 3, y, zg, a), pc.z, er, S.w,
                                      N.w, pm.w, pn.w, pc.w, vpp.w, c2w, vt.w, r3, a);
            st4(pp + o, out);
            if (zl == 0 && a.peer_lo) st4(a.peer_lo + row, out);
            if (zl + 1 == a.nz && a.peer_hi) st4(a.peer_hi + row, out);
        }

        if (more) {
            const int nxt = cur ^ 1;
            srow[nxt][w + 1][lane] = pn;
            if (ylo) srow[nxt][0][lane] = hy;
            if (yhi) srow[nxt][TY + 1][lane] = hy;
            if (xl) shl[nxt][w] = hx;
            if (xr) shr[nxt][w] = hx;
            __syncthreads();
            pm = pc; pc = pn; pn = pn2; vpp = vpp2; vc2 = vc22; vt = vt2;
            cur = nxt;
        }
    }
    // Order this thread's peer stores before the flag the signal raises.
    if ((a.peer_lo && zb == 0) || (a.peer_hi && ze == a.nz)) __threadfence_system();
    __syncthreads();
}

template <bool kC2F, bool kCells, int TY>
__global__ void __launch_bounds__(32 * TY, 3)
k_step_zstream(StepParams a, uint32_t zchunk) {
    const bool halo_wait = a.wait_lo != nullptr || a.wait_hi != nullptr;
    uint32_t zb, ze;
    zs_chunk(zs_chunk_order(blockIdx.z, gridDim.z, halo_wait), zchunk, a.nz, &zb, &ze);
    if (zb >= ze) return;  // uniform over the CTA, before any barrier
    zs_tile<kC2F, kCells, TY>(a, blockIdx.x, blockIdx.y, zb, ze);
}

// ---------------------------------------------------------------------------
// One thread per cell, boundary fused (comparator variant).
// ---------------------------------------------------------------------------
template <bool kC2F, bool kCells>
__global__ void __launch_bounds__(256) k_step_naive(StepParams a) {
    const uint32_t x = blockIdx.x * blockDim.x + threadIdx.x;
    const uint32_t y = blockIdx.y * blockDim.y + threadIdx.y;
    const uint32_t zl = blockIdx.z * blockDim.z + threadIdx.z;
    if (x >= a.W || y >= a.H || zl >= a.nz) return;
    const long long P = (long long)a.plane;
    const long long i = (long long)zl * P + (long long)y * a.pitch + x;
    const uint32_t zg = a.z0 + zl;
    const bool interior = is_interior(x, y, zg, a);
    uint8_t t = 0;
    float r = 0.f;
    if (kCells) {
        t = a.types[i];
        if (t == kAbsorber || t == kObstacle) r = a.refl[i];
    }
    float w = 0.f, e = 0.f, s = 0.f, n = 0.f, dn = 0.f, up = 0.f, c = 0.f;
    float c2 = kC2F ? a.c2f[i] : a.c2;
    if (interior) {
        c = a.p[i];
        w = a.p[i - 1]; e = a.p[i + 1];
        s = a.p[i - a.pitch]; n = a.p[i + a.pitch];
        dn = a.p[i - P]; up = a.p[i + P];
    }
    a.pp[i] = cell_rule<kCells>(x, y, zg, interior, w, e, s, n, dn, up, c, a.pp[i], c2, t, r, a);
}

// ---------------------------------------------------------------------------
// The reference's two-launch shape (gpu_backend.rs:27-100, :316-369): an
// 8x8x4-block stencil launch over interior Normal cells that reads the cell
// type of every cell, then a 1-D full-grid boundary launch.  Kept as the
// "reference kernels recompiled for sm_100a" comparator.
// ---------------------------------------------------------------------------
template <bool kC2F>
__global__ void __launch_bounds__(256) k_ref_stencil(StepParams a) {
    const uint32_t x = blockIdx.x * blockDim.x + threadIdx.x;
    const uint32_t y = blockIdx.y * blockDim.y + threadIdx.y;
    const uint32_t zl = blockIdx.z * blockDim.z + threadIdx.z;
    if (zl >= a.nz) return;
    const uint32_t zg = a.z0 + zl;
    if (!is_interior(x, y, zg, a)) return;
    const long long P = (long long)a.plane;
    const long long i = (long long)zl * P + (long long)y * a.pitch + x;
    if (a.types[i] != kNormal) return;
    const float c2 = kC2F ? a.c2f[i] : a.c2;
    float v = leapfrog(a.p[i - 1], a.p[i + 1], a.p[i - a.pitch], a.p[i + a.pitch], a.p[i - P],
                       a.p[i + P], a.p[i], a.pp[i], c2, a.damping);
    if (a.sponge_w) {
        uint32_t d = face_dist(x, y, zg, a);
        if (d < a.sponge_w) v = __fmul_rn(v, a.sponge[d]);
    }
    a.pp[i] = v;
}

__global__ void __launch_bounds__(256) k_ref_boundary(float* pp, const uint8_t* types,
                                                      const float* refl, uint64_t n) {
    const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const uint8_t t = types[i];
    if (t == kAbsorber || t == kObstacle) pp[i] = __fmul_rn(pp[i], refl[i]);
}

// ---------------------------------------------------------------------------
// Sources and impulses.
// ---------------------------------------------------------------------------

// Per-step point sources, applied in source order by one thread so that
// coinciding sources add in the same order as the reference loop.  A source
// on a plane that a neighbouring slab holds as a ghost plane also updates that
// copy: ghost_off[2k] / [2k+1] is the offset of source k's cell in the lower /
// upper neighbour's copy (relative to ghost_lo = its plane -1, ghost_hi = its
// plane -2), or -1 when that neighbour holds no copy of the cell.  A copy
// equals the cell, so the new value is stored (no read over NVLink).
__device__ __forceinline__ void inject_sources_dev(float* p, float* pp, const uint64_t* off,
                                                   const float* wavelet, uint32_t n, uint64_t len,
                                                   uint64_t step, const long long* ghost_off,
                                                   float* ghost_lo, float* ghost_hi) {
    for (uint32_t k = 0; k < n; ++k) {
        const float amp = step < len ? wavelet[(uint64_t)k * len + step] : 0.0f;
        p[off[k]] = __fadd_rn(p[off[k]], amp);
        pp[off[k]] = __fadd_rn(pp[off[k]], __fmul_rn(amp, 0.5f));
        if (ghost_off) {
            const long long gl = ghost_off[2 * k], gh = ghost_off[2 * k + 1];
            if (gl >= 0 && ghost_lo) ghost_lo[gl] = p[off[k]];
            if (gh >= 0 && ghost_hi) ghost_hi[gh] = p[off[k]];
        }
    }
}

// Sources of one step; on z-slabs also the halo signal of k_halo_signal
// (flags non-null), after the sources reached the neighbours' copies.
__global__ void k_inject_sources(float* p, float* pp, const uint64_t* off, const float* wavelet,
                                 uint32_t n, uint64_t len, uint64_t step,
                                 const long long* ghost_off, float* ghost_lo, float* ghost_hi,
                                 unsigned long long* flag_lo, unsigned long long* flag_hi,
                                 unsigned long long flag_val) {
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    inject_sources_dev(p, pp, off, wavelet, n, len, step, ghost_off, ghost_lo, ghost_hi);
    if (flag_lo || flag_hi) {
        __threadfence_system();
        if (flag_lo) st_release_sys(flag_lo, flag_val);
        if (flag_hi) st_release_sys(flag_hi, flag_val);
    }
}

// Impulse factors applied to a neighbour's ghost copy of a boundary plane
// (pressure only: ghost planes hold no p_prev).
__global__ void k_inject_ghost(float* ghost, const uint64_t* row, const float* factor, uint32_t n,
                               float amp) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    ghost[row[i]] = __fadd_rn(ghost[row[i]], __fmul_rn(amp, factor[i]));
}

// grid3d.rs:146-152 / gpu_backend.rs:118-131 (offset precomputed on the host).
__global__ void k_inject_point(float* p, float* pp, uint64_t off, float amp) {
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    p[off] = __fadd_rn(p[off], amp);
    pp[off] = __fadd_rn(pp[off], __fmul_rn(amp, 0.5f));
}

// grid3d.rs:161-191: one thread per affected cell (distinct offsets).
__global__ void k_inject_table(float* p, float* pp, const uint64_t* off, const float* factor,
                               uint32_t n, float amp) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float v = __fmul_rn(amp, factor[i]);
    p[off[i]] = __fadd_rn(p[off[i]], v);
    pp[off[i]] = __fadd_rn(pp[off[i]], __fmul_rn(v, 0.5f));
}

// ---------------------------------------------------------------------------
// Trilinear sampling (grid3d.rs:373-411), f32 in the reference order.  pos
// holds n (x, y, z) positions in metres; p addresses owned plane 0 of the
// current field; samples need planes z0 and z0+1 inside [0, nz] (plane nz is
// the upper ghost, valid on a synchronised slab).
// ---------------------------------------------------------------------------
__global__ void k_sample(const float* p, uint32_t W, uint32_t H, uint32_t Dg, uint32_t pitch,
                         uint64_t plane, uint32_t z_first, const float* pos, float cell_size,
                         uint32_t n, float* out) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float fx = __fdiv_rn(pos[3 * i + 0], cell_size);
    const float fy = __fdiv_rn(pos[3 * i + 1], cell_size);
    const float fz = __fdiv_rn(pos[3 * i + 2], cell_size);
    // `as usize` saturates negative values to 0
    const float flx = floorf(fx), fly = floorf(fy), flz = floorf(fz);
    const uint32_t x0 = flx > 0.f ? (uint32_t)flx : 0u;
    const uint32_t y0 = fly > 0.f ? (uint32_t)fly : 0u;
    const uint32_t z0 = flz > 0.f ? (uint32_t)flz : 0u;
    const uint32_t x1 = min(x0 + 1u, W - 1u), y1 = min(y0 + 1u, H - 1u), z1 = min(z0 + 1u, Dg - 1u);
    const float tx = __fsub_rn(fx, (float)x0), ty = __fsub_rn(fy, (float)y0);
    const float tz = __fsub_rn(fz, (float)z0);
    auto at = [&](uint32_t x, uint32_t y, uint32_t z) {
        return p[(int64_t)(z - z_first) * (int64_t)plane + (int64_t)y * pitch + x];
    };
    auto lerp = [](float a, float b, float t) {
        return __fadd_rn(__fmul_rn(a, __fsub_rn(1.0f, t)), __fmul_rn(b, t));
    };
    const float c00 = lerp(at(x0, y0, z0), at(x1, y0, z0), tx);
    const float c01 = lerp(at(x0, y0, z1), at(x1, y0, z1), tx);
    const float c10 = lerp(at(x0, y1, z0), at(x1, y1, z0), tx);
    const float c11 = lerp(at(x0, y1, z1), at(x1, y1, z1), tx);
    const float c0 = lerp(c00, c10, ty);
    const float c1 = lerp(c01, c11, ty);
    out[i] = lerp(c0, c1, tz);
}

// ---------------------------------------------------------------------------
// Reductions over the owned cells (padding excluded).  Deterministic: each
// block writes one partial into a scratch array; one block folds the
// partials in a fixed order.
// ---------------------------------------------------------------------------
constexpr int kRedThreads = 256;

__device__ __forceinline__ double warp_sum(double v) {
    for (int o = 16; o > 0; o >>= 1) v += __shfl_down_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_down_sync(0xffffffffu, v, o));
    return v;
}

// rows = nz * H rows of W valid floats, row pitch `pitch`.
__global__ void __launch_bounds__(kRedThreads) k_energy_partials(const float* p, uint32_t W,
                                                                 uint32_t pitch, uint64_t rows,
                                                                 double* partials) {
    __shared__ double sm[kRedThreads / 32];
    double acc = 0.0;
    const uint64_t nvec = rows * (pitch / 4);
    for (uint64_t v = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; v < nvec;
         v += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t r = v / (pitch / 4);
        const uint32_t x = (uint32_t)(v - r * (pitch / 4)) * 4u;
        if (x >= W) continue;
        const float4 q = ld4_stream(p + r * pitch + x);
        acc += (double)q.x * q.x;
        if (x + 1 < W) acc += (double)q.y * q.y;
        if (x + 2 < W) acc += (double)q.z * q.z;
        if (x + 3 < W) acc += (double)q.w * q.w;
    }
    acc = warp_sum(acc);
    if ((threadIdx.x & 31) == 0) sm[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x < 32) {
        double t = threadIdx.x < kRedThreads / 32 ? sm[threadIdx.x] : 0.0;
        t = warp_sum(t);
        if (threadIdx.x == 0) partials[blockIdx.x] = t;
    }
}

__global__ void __launch_bounds__(kRedThreads) k_fold_partials(const double* partials,
                                                               uint32_t n, double* out) {
    __shared__ double sm[kRedThreads / 32];
    double acc = 0.0;
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) acc += partials[i];
    acc = warp_sum(acc);
    if ((threadIdx.x & 31) == 0) sm[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x < 32) {
        double t = threadIdx.x < kRedThreads / 32 ? sm[threadIdx.x] : 0.0;
        t = warp_sum(t);
        if (threadIdx.x == 0) *out = t;
    }
}

__global__ void __launch_bounds__(kRedThreads) k_maxabs_partials(const float* p, uint32_t W,
                                                                 uint32_t pitch, uint64_t rows,
                                                                 float* partials) {
    __shared__ float sm[kRedThreads / 32];
    float acc = 0.f;
    const uint64_t nvec = rows * (pitch / 4);
    for (uint64_t v = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; v < nvec;
         v += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t r = v / (pitch / 4);
        const uint32_t x = (uint32_t)(v - r * (pitch / 4)) * 4u;
        if (x >= W) continue;
        const float4 q = ld4_stream(p + r * pitch + x);
        acc = fmaxf(acc, fabsf(q.x));
        if (x + 1 < W) acc = fmaxf(acc, fabsf(q.y));
        if (x + 2 < W) acc = fmaxf(acc, fabsf(q.z));
        if (x + 3 < W) acc = fmaxf(acc, fabsf(q.w));
    }
    acc = warp_max(acc);
    if ((threadIdx.x & 31) == 0) sm[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x < 32) {
        float t = threadIdx.x < kRedThreads / 32 ? sm[threadIdx.x] : 0.f;
        t = warp_max(t);
        if (threadIdx.x == 0) partials[blockIdx.x] = t;
    }
}

__global__ void __launch_bounds__(kRedThreads) k_fold_max(const float* partials, uint32_t n,
                                                          float* out) {
    __shared__ float sm[kRedThreads / 32];
    float acc = 0.f;
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) acc = fmaxf(acc, partials[i]);
    acc = warp_max(acc);
    if ((threadIdx.x & 31) == 0) sm[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x < 32) {
        float t = threadIdx.x < kRedThreads / 32 ? sm[threadIdx.x] : 0.f;
        t = warp_max(t);
        if (threadIdx.x == 0) *out = t;
    }
}

}  // namespace ws3d
