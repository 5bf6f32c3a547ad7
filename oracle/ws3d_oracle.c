/*
 * ws3d_oracle.c -- CPU restatement of the reference WaveSim3D FDTD step.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the shipped library links, loads or
 * calls this file.  It is the checker that the CUDA path is compared against
 * (tests/, __graft_entry__.smoke(), and the CPU-baseline leg of bench.py).
 *
 * Reference: mivertowski/RustCompute, crate ringkernel-wavesim3d,
 *   src/simulation/grid3d.rs
 *     :71-116   SimulationGrid3D::new / setup_boundaries (faces = Absorber, refl 0.1)
 *     :120-122  index = z*W*H + y*W + x (z-major, x fastest)
 *     :146-152  inject_impulse      p += a ; p_prev += a*0.5
 *     :161-191  inject_spherical_impulse  factor = exp(-d2 / (2 r))  (r, not r^2)
 *     :222-269  step_sequential     interior Normal cells, in-place into p_prev,
 *                                   lap = ((((W+E)+S)+N)+D)+U - 6p
 *                                   p_new = (2p - p_prev) + c2*lap ; p_prev = p_new*damping
 *     :272-350  step_parallel       same arithmetic, z-planes in parallel
 *     :353-370  apply_boundary_conditions  Absorber/Obstacle: p_prev *= refl
 *     :264-268  swap(pressure, pressure_prev), step += 1
 *     :445-455  total_energy / max_pressure
 *
 * Parity status: the reference's Rust crate cannot be built in this image
 * (no cargo/rustc, and the crate hard-depends on wgpu).  This restatement is
 * pinned by the reference's own known-answer tests (restated in
 * tests/test_oracle.py: indexing, impulse injection, boundary setup, slices,
 * parallel-vs-sequential, wave spreading) and by an analytic discrete
 * eigenmode solution of the same leapfrog scheme.  No field dump produced by
 * the reference itself exists, so parity against the reference's own output is
 * "pinned by known-answer tests only".
 *
 * Extensions beyond the reference CPU path (used by the larger configs; the
 * reference never implemented them, so their parity is unpinned except that
 * each reduces bit-for-bit to the plain restatement when switched off):
 *   - per-cell Courant^2 field c2[idx] replacing the scalar c_squared
 *   - sponge multiplier s(d), d = distance to the nearest face, applied right
 *     after the reference's `* damping`:  out = (p_new*damping)*s(d), d < w
 *   - additive point sources with the inject_impulse semantic, applied before
 *     each step:  p[i] += a(step) ; p_prev[i] += a(step)*0.5
 *
 * Build: gcc -O3 -ffp-contract=off -fno-fast-math -fopenmp (oracle/Makefile).
 * -ffp-contract=off keeps every multiply and add separately rounded, which is
 * the semantics of the Rust source (Rust never contracts to FMA).
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* CellType discriminants as uploaded by the reference GPU backend
 * (gpu_backend.rs:261-270). */
enum { CT_NORMAL = 0, CT_ABSORBER = 1, CT_REFLECTOR = 2, CT_OBSTACLE = 3 };

typedef struct {
    float c_squared;        /* scalar Courant^2 (grid3d.rs:223) */
    float damping;          /* simple_damping (grid3d.rs:224)  */
    const float *c2_field;  /* optional per-cell Courant^2, NULL = scalar */
    const float *sponge;    /* optional table s[d], d in [0, sponge_w) */
    uint32_t sponge_w;      /* 0 = no sponge */
} ws3o_params;

static inline size_t IDX(size_t W, size_t H, size_t x, size_t y, size_t z) {
    return z * (W * H) + y * W + x;
}

/* grid3d.rs:96-116 */
void ws3o_setup_boundaries(uint32_t W, uint32_t H, uint32_t D,
                           uint8_t *types, float *refl) {
    for (size_t z = 0; z < D; ++z)
        for (size_t y = 0; y < H; ++y)
            for (size_t x = 0; x < W; ++x) {
                size_t i = IDX(W, H, x, y, z);
                int face = x == 0 || x == W - 1 || y == 0 || y == H - 1 ||
                           z == 0 || z == D - 1;
                types[i] = face ? CT_ABSORBER : CT_NORMAL;
                refl[i] = face ? 0.1f : 1.0f;
            }
}

/* grid3d.rs:146-152 */
void ws3o_inject_impulse(uint32_t W, uint32_t H, uint32_t D, float *p, float *pp,
                         uint32_t x, uint32_t y, uint32_t z, float amp) {
    if (x < W && y < H && z < D) {
        size_t i = IDX(W, H, x, y, z);
        p[i] += amp;
        pp[i] += amp * 0.5f;
    }
}

/* grid3d.rs:161-191, with the centre already converted to grid indices. */
void ws3o_inject_spherical(uint32_t W, uint32_t H, uint32_t D, float *p, float *pp,
                           uint32_t cx, uint32_t cy, uint32_t cz, float amp,
                           float radius) {
    int r = (int)radius;
    float r_sq = radius * radius;
    for (int dz = -r; dz <= r; ++dz)
        for (int dy = -r; dy <= r; ++dy)
            for (int dx = -r; dx <= r; ++dx) {
                int x = (int)cx + dx, y = (int)cy + dy, z = (int)cz + dz;
                if (x < 0 || y < 0 || z < 0 || x >= (int)W || y >= (int)H ||
                    z >= (int)D)
                    continue;
                float dist_sq = (float)(dx * dx + dy * dy + dz * dz);
                if (dist_sq <= r_sq) {
                    float factor = expf(-dist_sq / (2.0f * radius));
                    size_t i = IDX(W, H, (size_t)x, (size_t)y, (size_t)z);
                    p[i] += amp * factor;
                    pp[i] += amp * factor * 0.5f;
                }
            }
}

/* Sponge table: s(d) = 1 - smax*((w-d)/w)^2 for d in [0, w), evaluated in
 * double and rounded once to f32. */
void ws3o_sponge_table(uint32_t w, float smax, float *out) {
    for (uint32_t d = 0; d < w; ++d) {
        double t = (double)(w - d) / (double)w;
        out[d] = (float)(1.0 - (double)smax * t * t);
    }
}

static inline uint32_t min_u32(uint32_t a, uint32_t b) { return a < b ? a : b; }

/* Distance of a cell to the nearest face, in cells. */
static inline uint32_t face_dist(uint32_t W, uint32_t H, uint32_t D, uint32_t x,
                                 uint32_t y, uint32_t z) {
    uint32_t d = min_u32(x, W - 1 - x);
    d = min_u32(d, min_u32(y, H - 1 - y));
    d = min_u32(d, min_u32(z, D - 1 - z));
    return d;
}

/* One interior cell, reference operation order (grid3d.rs:238-256). */
static inline float cell_update(const float *p, const float *pp, size_t i, size_t W,
                                size_t S, float c2, float damping) {
    float pc = p[i];
    float pprev = pp[i];
    float p_west = p[i - 1];
    float p_east = p[i + 1];
    float p_south = p[i - W];
    float p_north = p[i + W];
    float p_down = p[i - S];
    float p_up = p[i + S];
    float lap = p_west + p_east + p_south + p_north + p_down + p_up - 6.0f * pc;
    float p_new = 2.0f * pc - pprev + c2 * lap;
    return p_new * damping;
}

/* Interior update of one z-plane, in place into pp (grid3d.rs:227-259). */
static void plane_update(uint32_t W, uint32_t H, uint32_t D, const float *p, float *pp,
                         const uint8_t *types, const ws3o_params *prm, uint32_t z) {
    const size_t S = (size_t)W * H;
    for (uint32_t y = 1; y + 1 < H; ++y)
        for (uint32_t x = 1; x + 1 < W; ++x) {
            size_t i = IDX(W, H, x, y, z);
            if (types && types[i] != CT_NORMAL) continue;
            float c2 = prm->c2_field ? prm->c2_field[i] : prm->c_squared;
            float v = cell_update(p, pp, i, W, S, c2, prm->damping);
            if (prm->sponge_w) {
                uint32_t d = face_dist(W, H, D, x, y, z);
                if (d < prm->sponge_w) v = v * prm->sponge[d];
            }
            pp[i] = v;
        }
}

/* grid3d.rs:353-370.  types == NULL means the default layout of
 * setup_boundaries (faces Absorber with refl 0.1, interior Normal). */
static void boundary_pass(uint32_t W, uint32_t H, uint32_t D, float *pp,
                          const uint8_t *types, const float *refl, int nthreads) {
    const size_t N = (size_t)W * H * D;
    if (types) {
#pragma omp parallel for schedule(static) num_threads(nthreads) if (nthreads > 1)
        for (size_t i = 0; i < N; ++i) {
            uint8_t t = types[i];
            if (t == CT_ABSORBER || t == CT_OBSTACLE) pp[i] *= refl[i];
        }
        return;
    }
#pragma omp parallel for schedule(static) num_threads(nthreads) if (nthreads > 1)
    for (uint32_t z = 0; z < D; ++z)
        for (uint32_t y = 0; y < H; ++y) {
            size_t row = IDX(W, H, 0, y, z);
            if (z == 0 || z == D - 1 || y == 0 || y == H - 1) {
                for (uint32_t x = 0; x < W; ++x) pp[row + x] *= 0.1f;
            } else {
                pp[row] *= 0.1f;
                if (W > 1) pp[row + W - 1] *= 0.1f;
            }
        }
}

/* step_sequential minus the swap: writes the new field into pp. */
void ws3o_step_sequential(uint32_t W, uint32_t H, uint32_t D, const float *p, float *pp,
                          const uint8_t *types, const float *refl,
                          const ws3o_params *prm) {
    if (W < 3 || H < 3 || D < 3) {
        boundary_pass(W, H, D, pp, types, refl, 1);
        return;
    }
    for (uint32_t z = 1; z + 1 < D; ++z) plane_update(W, H, D, p, pp, types, prm, z);
    boundary_pass(W, H, D, pp, types, refl, 1);
}

/* step_parallel minus the swap (grid3d.rs:272-350).  The reference computes
 * interior planes into a scratch buffer in parallel and copies back; since a
 * cell reads only its own p_prev entry and p is read-only during the step,
 * updating in place per plane gives the identical result. */
void ws3o_step_parallel(uint32_t W, uint32_t H, uint32_t D, const float *p, float *pp,
                        const uint8_t *types, const float *refl,
                        const ws3o_params *prm, int nthreads) {
    if (W < 3 || H < 3 || D < 3) {
        boundary_pass(W, H, D, pp, types, refl, nthreads);
        return;
    }
#pragma omp parallel for schedule(static) num_threads(nthreads) if (nthreads > 1)
    for (uint32_t z = 1; z < D - 1; ++z) plane_update(W, H, D, p, pp, types, prm, z);
    boundary_pass(W, H, D, pp, types, refl, nthreads);
}

/* Run `nsteps` steps starting at global step `step0`.
 *
 * p / pp hold the current and previous field on entry and on return (the
 * function swaps internally and copies back when the step count is odd, so
 * the caller's arrays play the roles of grid.pressure / grid.pressure_prev).
 * Sources: before each step s, for every source k,
 *   a = (s < wl_len) ? wavelet[k*wl_len + s] : 0 ;  p[i] += a ; pp[i] += a*0.5
 * (inject_impulse semantic, grid3d.rs:146-152, driven per step the way
 * bin/wavesim3d.rs:80-100 drives it).  nthreads <= 1 selects step_sequential.
 */
/* ws3o_run without the copy-back: returns 1 when the current field ends in
 * pp (odd nsteps), 0 when it ends in p; the caller swaps its references, as
 * the reference swaps its buffers (grid3d.rs:264). */
int ws3o_run_swap(uint32_t W, uint32_t H, uint32_t D, float *p, float *pp,
                  const uint8_t *types, const float *refl, const ws3o_params *prm,
                  uint64_t step0, uint64_t nsteps, uint32_t n_src, const uint64_t *src_idx,
                  const float *wavelet, uint64_t wl_len, int nthreads) {
    float *cur = p, *prev = pp;
    for (uint64_t s = 0; s < nsteps; ++s) {
        uint64_t gs = step0 + s;
        for (uint32_t k = 0; k < n_src; ++k) {
            float a = gs < wl_len ? wavelet[(size_t)k * wl_len + gs] : 0.0f;
            cur[src_idx[k]] += a;
            prev[src_idx[k]] += a * 0.5f;
        }
        if (nthreads > 1)
            ws3o_step_parallel(W, H, D, cur, prev, types, refl, prm, nthreads);
        else
            ws3o_step_sequential(W, H, D, cur, prev, types, refl, prm);
        float *t = cur; cur = prev; prev = t;
    }
    return cur != p;
}

void ws3o_run(uint32_t W, uint32_t H, uint32_t D, float *p, float *pp,
              const uint8_t *types, const float *refl, const ws3o_params *prm,
              uint64_t step0, uint64_t nsteps, uint32_t n_src, const uint64_t *src_idx,
              const float *wavelet, uint64_t wl_len, int nthreads) {
    float *cur = p, *prev = pp;
    for (uint64_t s = 0; s < nsteps; ++s) {
        uint64_t gs = step0 + s;
        for (uint32_t k = 0; k < n_src; ++k) {
            float a = gs < wl_len ? wavelet[(size_t)k * wl_len + gs] : 0.0f;
            cur[src_idx[k]] += a;
            prev[src_idx[k]] += a * 0.5f;
        }
        if (nthreads > 1)
            ws3o_step_parallel(W, H, D, cur, prev, types, refl, prm, nthreads);
        else
            ws3o_step_sequential(W, H, D, cur, prev, types, refl, prm);
        float *t = cur; cur = prev; prev = t;
    }
    if (cur != p) {
        size_t N = (size_t)W * H * D;
        float *tmp = (float *)malloc(N * sizeof(float));
        memcpy(tmp, p, N * sizeof(float));
        memcpy(p, cur, N * sizeof(float));
        memcpy(pp, tmp, N * sizeof(float));
        free(tmp);
    }
}

/* grid3d.rs:445-455 (sum in f32 in index order, like Iterator::sum) */
float ws3o_total_energy_f32(const float *p, uint64_t n) {
    float s = 0.0f;
    for (uint64_t i = 0; i < n; ++i) s += p[i] * p[i];
    return s;
}

double ws3o_total_energy_f64(const float *p, uint64_t n) {
    double s = 0.0;
    for (uint64_t i = 0; i < n; ++i) s += (double)p[i] * (double)p[i];
    return s;
}

float ws3o_max_pressure(const float *p, uint64_t n) {
    float m = 0.0f;
    for (uint64_t i = 0; i < n; ++i) {
        float a = fabsf(p[i]);
        if (a > m) m = a;
    }
    return m;
}

int ws3o_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* ---------------------------------------------------------------------------
 * Volume ray-march (visualization/volume.rs:76-160 shader, :396-420
 * update_volume; camera camera.rs:51-61, 98-110), restated on the CPU with
 * the operations of the CUDA renderer in the same order, so that the images
 * agree bit for bit.  Test infrastructure only.
 * ------------------------------------------------------------------------- */
typedef struct {
    uint32_t width, height;
    float density_scale, step_size;
    uint32_t max_steps;
    float threshold, cell_size, fov_y;
    float eye[3], target[3], up[3];
    uint32_t default_camera;
    float background[4];
    uint32_t composite;
    uint32_t reserved[3];
} ws3o_volume_params;

/* IEEE binary16 round-to-nearest-even (the half crate's f16::from_f32 and
 * CUDA's __float2half_rn); finite inputs of magnitude <= 65504 suffice here. */
static uint16_t f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t ex = (x >> 23) & 0xffu;
    uint32_t mant = x & 0x7fffffu;
    if (ex == 0xffu) return (uint16_t)(sign | 0x7c00u | (mant ? 0x200u : 0u));
    const int e = (int)ex - 127 + 15;
    if (e >= 31) return (uint16_t)(sign | 0x7c00u);
    if (e <= 0) {
        if (e < -10) return (uint16_t)sign;
        mant |= 0x800000u;
        const int shift = 14 - e;
        uint32_t h = mant >> shift;
        const uint32_t rem = mant & ((1u << shift) - 1u), halfway = 1u << (shift - 1);
        if (rem > halfway || (rem == halfway && (h & 1u))) ++h;
        return (uint16_t)(sign | h);
    }
    uint32_t h = sign | ((uint32_t)e << 10) | (mant >> 13);
    const uint32_t rem = mant & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) ++h;
    return (uint16_t)h;
}

static float f16_to_f32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    const uint32_t ex = (h >> 10) & 0x1fu, mant = h & 0x3ffu;
    uint32_t x;
    if (ex == 0) {
        if (mant == 0) {
            x = sign;
        } else {  /* subnormal: mant * 2^-24, exact in f32 */
            float v = (float)mant * 5.9604644775390625e-8f;
            memcpy(&x, &v, 4);
            x |= sign;
        }
    } else if (ex == 31) {
        x = sign | 0x7f800000u | (mant << 13);
    } else {
        x = sign | ((ex - 15 + 127) << 23) | (mant << 13);
    }
    float f;
    memcpy(&f, &x, 4);
    return f;
}

static float lerp_rn(float a, float b, float t) { return a * (1.0f - t) + b * t; }

static float vol_sample(const float *vol, uint32_t W, uint32_t H, uint32_t D, float u, float w_,
                        float s) {
    const float cx = u * (float)W - 0.5f, cy = w_ * (float)H - 0.5f, cz = s * (float)D - 0.5f;
    const float x0f = floorf(cx), y0f = floorf(cy), z0f = floorf(cz);
    const float fx = cx - x0f, fy = cy - y0f, fz = cz - z0f;
    const int x0 = (int)x0f, y0 = (int)y0f, z0 = (int)z0f;
#define CL(v, n) ((v) < 0 ? 0 : ((v) > (int)(n) - 1 ? (int)(n) - 1 : (v)))
    const int xa = CL(x0, W), xb = CL(x0 + 1, W), ya = CL(y0, H), yb = CL(y0 + 1, H);
    const int za = CL(z0, D), zb = CL(z0 + 1, D);
#undef CL
#define V(x, y, z) vol[((size_t)(z) * H + (y)) * W + (x)]
    const float c00 = lerp_rn(V(xa, ya, za), V(xb, ya, za), fx);
    const float c10 = lerp_rn(V(xa, yb, za), V(xb, yb, za), fx);
    const float c01 = lerp_rn(V(xa, ya, zb), V(xb, ya, zb), fx);
    const float c11 = lerp_rn(V(xa, yb, zb), V(xb, yb, zb), fx);
#undef V
    return lerp_rn(lerp_rn(c00, c10, fy), lerp_rn(c01, c11, fy), fz);
}

/* p: W x H x D z-major field; rgba: width x height x 4.  Returns 0 or -1
 * (eye == target, or up parallel to the view). */
int ws3o_render_volume(const float *p, uint32_t W, uint32_t H, uint32_t D,
                       const ws3o_volume_params *prm, float *rgba) {
    const size_t n = (size_t)W * H * D;
    float mx = 0.0f;
    for (size_t i = 0; i < n; ++i) mx = fmaxf(mx, fabsf(p[i]));
    const float m = fmaxf(mx, 0.001f);
    float *vol = (float *)malloc(n * sizeof(float));
    if (!vol) return -1;
    for (size_t i = 0; i < n; ++i) vol[i] = f16_to_f32(f32_to_f16(p[i] / m));

    const float gx = (float)W * prm->cell_size, gy = (float)H * prm->cell_size;
    const float gz = (float)D * prm->cell_size;
    float eye[3], tgt[3];
    if (prm->default_camera) {
        const float cx = gx / 2.0f, cy = gy / 2.0f, cz = gz / 2.0f;
        const float dist = fmaxf(fmaxf(gx, gz) * 1.5f, 5.0f);
        eye[0] = cx + dist;
        eye[1] = cy + dist * 0.7f;
        eye[2] = cz + dist;
        tgt[0] = cx;
        tgt[1] = cy;
        tgt[2] = cz;
    } else {
        for (int k = 0; k < 3; ++k) {
            eye[k] = prm->eye[k];
            tgt[k] = prm->target[k];
        }
    }
    float f[3] = {tgt[0] - eye[0], tgt[1] - eye[1], tgt[2] - eye[2]};
    float len = sqrtf(f[0] * f[0] + f[1] * f[1] + f[2] * f[2]);
    if (!(len > 0.0f)) {
        free(vol);
        return -1;
    }
    for (int k = 0; k < 3; ++k) f[k] = f[k] / len;
    const float *up = prm->up;
    float r[3] = {f[1] * up[2] - f[2] * up[1], f[2] * up[0] - f[0] * up[2],
                  f[0] * up[1] - f[1] * up[0]};
    len = sqrtf(r[0] * r[0] + r[1] * r[1] + r[2] * r[2]);
    if (!(len > 0.0f)) {
        free(vol);
        return -1;
    }
    for (int k = 0; k < 3; ++k) r[k] = r[k] / len;
    const float u[3] = {r[1] * f[2] - r[2] * f[1], r[2] * f[0] - r[0] * f[2],
                        r[0] * f[1] - r[1] * f[0]};
    const float tan_half = (float)tan((double)prm->fov_y * 0.5);
    const float aspect = (float)prm->width / (float)prm->height;
    const float bmax[3] = {gx, gy, gz};

    for (uint32_t j = 0; j < prm->height; ++j)
        for (uint32_t i = 0; i < prm->width; ++i) {
            const float xn = ((2.0f * ((float)i + 0.5f)) / (float)prm->width - 1.0f) * tan_half *
                             aspect;
            const float yn = (1.0f - (2.0f * ((float)j + 0.5f)) / (float)prm->height) * tan_half;
            float d[3];
            for (int k = 0; k < 3; ++k) d[k] = (f[k] + r[k] * xn) + u[k] * yn;
            const float dl = sqrtf((d[0] * d[0] + d[1] * d[1]) + d[2] * d[2]);
            for (int k = 0; k < 3; ++k) d[k] = d[k] / dl;
            float tn = -INFINITY, tf = INFINITY;
            for (int k = 0; k < 3; ++k) {
                const float inv = 1.0f / d[k];
                const float t1 = (0.0f - eye[k]) * inv, t2 = (bmax[k] - eye[k]) * inv;
                tn = fmaxf(tn, fminf(t1, t2));
                tf = fminf(tf, fmaxf(t1, t2));
            }
            float acc[4] = {0.f, 0.f, 0.f, 0.f};
            int hit = !(tn > tf || tf < 0.0f);
            if (hit) {
                float t = fmaxf(tn, 0.0f);
                for (uint32_t steps = 0; !(t >= tf || steps >= prm->max_steps || acc[3] >= 0.95f);
                     ++steps) {
                    float uvw[3];
                    for (int k = 0; k < 3; ++k) uvw[k] = (eye[k] + d[k] * t) / bmax[k];
                    const float pr = vol_sample(vol, W, H, D, uvw[0], uvw[1], uvw[2]);
                    if (fabsf(pr) > prm->threshold) {
                        const float pc = fminf(fmaxf(pr, -1.0f), 1.0f);
                        float cr, cg, cb;
                        if (pc >= 0.0f) {
                            cr = 1.0f;
                            cg = 1.0f - pc;
                            cb = 1.0f - pc;
                        } else {
                            cr = 1.0f + pc;
                            cg = 1.0f + pc;
                            cb = 1.0f;
                        }
                        const float sa = fabsf(pc) * prm->density_scale;
                        const float alpha = sa * (1.0f - acc[3]);
                        acc[0] = acc[0] + cr * alpha;
                        acc[1] = acc[1] + cg * alpha;
                        acc[2] = acc[2] + cb * alpha;
                        acc[3] = acc[3] + alpha;
                    }
                    t = t + prm->step_size;
                }
                if (acc[3] < 0.01f) hit = 0;
            }
            float *o = rgba + ((size_t)j * prm->width + i) * 4;
            if (!hit) acc[0] = acc[1] = acc[2] = acc[3] = 0.0f;
            if (prm->composite) {
                if (!hit) {
                    for (int k = 0; k < 4; ++k) o[k] = prm->background[k];
                } else {
                    const float ia = 1.0f - acc[3];
                    for (int k = 0; k < 3; ++k) o[k] = acc[k] * acc[3] + prm->background[k] * ia;
                    o[3] = acc[3] + prm->background[3] * ia;
                }
            } else {
                for (int k = 0; k < 4; ++k) o[k] = acc[k];
            }
        }
    free(vol);
    return 0;
}

/* f32 -> f16 (round to nearest even) -> f32, for tests of the quantiser. */
void ws3o_quantize_f16(const float *in, uint64_t n, float *out) {
    for (uint64_t i = 0; i < n; ++i) out[i] = f16_to_f32(f32_to_f16(in[i]));
}
