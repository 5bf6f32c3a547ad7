// ws3d_volume.cuh -- headless volume ray-march of the pressure field.
//
// Restates the reference's volume renderer (crates/ringkernel-wavesim3d/src/
// visualization/volume.rs): update_volume (:396-420) normalises the pressure
// by max(max|p|, 0.001) and stores it as f16; the fragment shader (:103-160)
// marches each pixel's ray through the box [0, grid_size] in steps of
// step_size, samples the volume with linear filtering and clamp-to-edge,
// maps |p| > threshold to blue-white-red with alpha |p| * density_scale and
// composites front to back until alpha >= 0.95; pixels with alpha < 0.01
// are discarded.  Here there is no graphics pipeline: one thread per pixel
// computes the pixel's primary ray from the camera (the ray the rasterised
// proxy cube would carry, camera.rs look_at_rh / perspective_rh) and writes
// RGBA floats into a device buffer.  The texture filtering is done in
// software (texel centres at (i + 0.5) / N, weights in f32) so that every
// operation is a separately rounded f32 operation and a CPU restatement
// reproduces the image bit for bit.
#pragma once

#include <cuda_fp16.h>

#include "ws3d_kernels.cuh"

namespace ws3d {

struct VolumeArgs {
    const __half* vol;       // W x H x D normalised f16 values, z-major
    uint32_t W, H, D;
    float gx, gy, gz;        // grid_size (world units)
    float eye[3], fwd[3], right[3], upv[3];  // camera basis (unit vectors)
    float tan_half, aspect;  // tan(fov_y / 2), width / height
    float density_scale, step_size, threshold;
    uint32_t max_steps;
    uint32_t width, height;
    float bg[4];
    uint32_t composite;      // 0: fragment output (discarded = 0), 1: ALPHA_BLENDING over bg
    float4* out;             // width x height RGBA
};

// volume.rs:396-420: p / max(max|p|, 0.001) as f16 (round to nearest even).
__global__ void k_volume_normalize(const float* p, uint32_t W, uint32_t H, uint32_t D,
                                   uint32_t pitch, uint64_t plane, const float* maxabs,
                                   __half* vol) {
    const uint64_t n = (uint64_t)W * H * D;
    const float m = fmaxf(*maxabs, 0.001f);
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n;
         i += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t z = i / ((uint64_t)W * H), r = i - z * W * H, y = r / W, x = r - y * W;
        vol[i] = __float2half_rn(__fdiv_rn(p[z * plane + y * pitch + x], m));
    }
}

__device__ __forceinline__ float vol_at(const VolumeArgs& v, int x, int y, int z) {
    return __half2float(v.vol[((uint64_t)z * v.H + y) * v.W + x]);
}

__device__ __forceinline__ float lerp_rn(float a, float b, float t) {
    return __fadd_rn(__fmul_rn(a, __fsub_rn(1.0f, t)), __fmul_rn(b, t));
}

// textureSample with a linear filter and clamp-to-edge addressing.
__device__ __forceinline__ float sample_linear(const VolumeArgs& v, float u, float w_, float s) {
    const float cx = __fsub_rn(__fmul_rn(u, (float)v.W), 0.5f);
    const float cy = __fsub_rn(__fmul_rn(w_, (float)v.H), 0.5f);
    const float cz = __fsub_rn(__fmul_rn(s, (float)v.D), 0.5f);
    const float x0f = floorf(cx), y0f = floorf(cy), z0f = floorf(cz);
    const float fx = __fsub_rn(cx, x0f), fy = __fsub_rn(cy, y0f), fz = __fsub_rn(cz, z0f);
    const int x0 = (int)x0f, y0 = (int)y0f, z0 = (int)z0f;
    const int xa = min(max(x0, 0), (int)v.W - 1), xb = min(max(x0 + 1, 0), (int)v.W - 1);
    const int ya = min(max(y0, 0), (int)v.H - 1), yb = min(max(y0 + 1, 0), (int)v.H - 1);
    const int za = min(max(z0, 0), (int)v.D - 1), zb = min(max(z0 + 1, 0), (int)v.D - 1);
    const float c00 = lerp_rn(vol_at(v, xa, ya, za), vol_at(v, xb, ya, za), fx);
    const float c10 = lerp_rn(vol_at(v, xa, yb, za), vol_at(v, xb, yb, za), fx);
    const float c01 = lerp_rn(vol_at(v, xa, ya, zb), vol_at(v, xb, ya, zb), fx);
    const float c11 = lerp_rn(vol_at(v, xa, yb, zb), vol_at(v, xb, yb, zb), fx);
    return lerp_rn(lerp_rn(c00, c10, fy), lerp_rn(c01, c11, fy), fz);
}

__global__ void k_volume_render(VolumeArgs v) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    const uint32_t j = blockIdx.y * blockDim.y + threadIdx.y;
    if (i >= v.width || j >= v.height) return;
    // primary ray through the pixel centre
    const float xn = __fmul_rn(
        __fmul_rn(__fsub_rn(__fdiv_rn(__fmul_rn(2.0f, __fadd_rn((float)i, 0.5f)), (float)v.width),
                            1.0f),
                  v.tan_half),
        v.aspect);
    const float yn = __fmul_rn(
        __fsub_rn(1.0f,
                  __fdiv_rn(__fmul_rn(2.0f, __fadd_rn((float)j, 0.5f)), (float)v.height)),
        v.tan_half);
    float d[3];
    for (int k = 0; k < 3; ++k)
        d[k] = __fadd_rn(__fadd_rn(v.fwd[k], __fmul_rn(v.right[k], xn)), __fmul_rn(v.upv[k], yn));
    const float len = __fsqrt_rn(
        __fadd_rn(__fadd_rn(__fmul_rn(d[0], d[0]), __fmul_rn(d[1], d[1])), __fmul_rn(d[2], d[2])));
    for (int k = 0; k < 3; ++k) d[k] = __fdiv_rn(d[k], len);

    // intersect_box (volume.rs:89-101)
    const float bmax[3] = {v.gx, v.gy, v.gz};
    float tn = -INFINITY, tf = INFINITY;
    for (int k = 0; k < 3; ++k) {
        const float inv = __fdiv_rn(1.0f, d[k]);
        const float t1 = __fmul_rn(__fsub_rn(0.0f, v.eye[k]), inv);
        const float t2 = __fmul_rn(__fsub_rn(bmax[k], v.eye[k]), inv);
        tn = fmaxf(tn, fminf(t1, t2));
        tf = fminf(tf, fmaxf(t1, t2));
    }
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    bool hit = !(tn > tf || tf < 0.0f);
    if (hit) {
        float t = fmaxf(tn, 0.0f);
        for (uint32_t steps = 0; !(t >= tf || steps >= v.max_steps || acc.w >= 0.95f); ++steps) {
            float uvw[3];
            for (int k = 0; k < 3; ++k)
                uvw[k] = __fdiv_rn(__fadd_rn(v.eye[k], __fmul_rn(d[k], t)), bmax[k]);
            const float pr = sample_linear(v, uvw[0], uvw[1], uvw[2]);
            if (fabsf(pr) > v.threshold) {
                // pressure_to_color (volume.rs:104-115)
                const float p = fminf(fmaxf(pr, -1.0f), 1.0f);
                float r, g, b;
                if (p >= 0.0f) {
                    r = 1.0f;
                    g = __fsub_rn(1.0f, p);
                    b = __fsub_rn(1.0f, p);
                } else {
                    r = __fadd_rn(1.0f, p);
                    g = __fadd_rn(1.0f, p);
                    b = 1.0f;
                }
                const float sa = __fmul_rn(fabsf(p), v.density_scale);
                const float alpha = __fmul_rn(sa, __fsub_rn(1.0f, acc.w));
                acc.x = __fadd_rn(acc.x, __fmul_rn(r, alpha));
                acc.y = __fadd_rn(acc.y, __fmul_rn(g, alpha));
                acc.z = __fadd_rn(acc.z, __fmul_rn(b, alpha));
                acc.w = __fadd_rn(acc.w, alpha);
            }
            t = __fadd_rn(t, v.step_size);
        }
        if (acc.w < 0.01f) hit = false;  // discard
    }
    if (!hit) acc = make_float4(0.f, 0.f, 0.f, 0.f);
    float4 o = acc;
    if (v.composite) {  // BlendState::ALPHA_BLENDING over the cleared target
        if (!hit) {
            o = make_float4(v.bg[0], v.bg[1], v.bg[2], v.bg[3]);
        } else {
            const float ia = __fsub_rn(1.0f, acc.w);
            o.x = __fadd_rn(__fmul_rn(acc.x, acc.w), __fmul_rn(v.bg[0], ia));
            o.y = __fadd_rn(__fmul_rn(acc.y, acc.w), __fmul_rn(v.bg[1], ia));
            o.z = __fadd_rn(__fmul_rn(acc.z, acc.w), __fmul_rn(v.bg[2], ia));
            o.w = __fadd_rn(acc.w, __fmul_rn(v.bg[3], ia));
        }
    }
    v.out[(uint64_t)j * v.width + i] = o;
}

}  // namespace ws3d
