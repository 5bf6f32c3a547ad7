// ws3d_api.cu -- host side of libws3d.so: the C-ABI declared in include/ws3d.h.
//
// The context mirrors GpuBackend3D (crates/ringkernel-wavesim3d/src/simulation/
// gpu_backend.rs:172-494): it owns the device fields, launches the step and
// keeps the buffer roles (pressure / pressure_prev) by swapping indices
// instead of copying, exactly like gpu_backend.rs:372.
#include "ws3d.h"
#include "ws3d_kernels.cuh"

#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

using namespace ws3d;

struct ws3d_ctx {
    ws3d_desc desc{};
    uint32_t W = 0, H = 0, Dg = 0, z0 = 0, nz = 0, pitch = 0;
    size_t plane = 0;       // H * pitch floats
    size_t slab = 0;        // (nz + 2) * plane floats (ghost below + owned + ghost above)
    float* buf[2] = {nullptr, nullptr};
    int cur = 0;            // buf[cur] = pressure, buf[cur ^ 1] = pressure_prev
    float* c2f = nullptr;   // slab-shaped, or nullptr
    uint8_t* types = nullptr;
    float* refl = nullptr;
    bool cells_default = true;     // kernels evaluate the default face layout analytically
    bool types_hold_default = false;  // types/refl arrays currently hold that default layout
    float* sponge = nullptr;
    uint32_t sponge_w = 0;
    uint64_t* src_off = nullptr;
    float* wavelet = nullptr;
    uint32_t n_src = 0;
    uint64_t wl_len = 0;
    double* red_scratch = nullptr;  // reduction partials + result
    uint32_t red_blocks = 0;
    cudaStream_t own_stream = nullptr;
    cudaStream_t stream = nullptr;
    uint64_t step = 0;
    uint64_t launches = 0;
    size_t device_bytes = 0;
    int sm_count = 0;
    std::string err;
};

namespace {

struct DeviceGuard {
    int prev = -1;
    bool ok = true;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != dev) ok = cudaSetDevice(dev) == cudaSuccess;
    }
    ~DeviceGuard() {
        if (prev >= 0) cudaSetDevice(prev);
    }
};

ws3d_status fail(ws3d_ctx* c, ws3d_status s, const char* fmt, ...) {
    if (c) {
        char buf[512];
        va_list ap;
        va_start(ap, fmt);
        vsnprintf(buf, sizeof buf, fmt, ap);
        va_end(ap);
        c->err = buf;
    }
    return s;
}

ws3d_status cuda_fail(ws3d_ctx* c, ws3d_status s, cudaError_t e, const char* what) {
    return fail(c, s, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

#define WS3D_CUDA(ctx, call, status)                                  \
    do {                                                              \
        cudaError_t e_ = (call);                                      \
        if (e_ != cudaSuccess) return cuda_fail(ctx, status, e_, #call); \
    } while (0)

ws3d_status check_launch(ws3d_ctx* c, const char* what) {
    cudaError_t e = cudaGetLastError();
    if (e == cudaErrorNoKernelImageForDevice || e == cudaErrorInvalidDeviceFunction)
        return cuda_fail(c, WS3D_ECOMPILE, e, what);
    if (e != cudaSuccess) return cuda_fail(c, WS3D_ELAUNCH, e, what);
    c->launches++;
    return WS3D_OK;
}

template <class T>
ws3d_status dalloc(ws3d_ctx* c, T** p, size_t count, const char* what) {
    void* q = nullptr;
    cudaError_t e = cudaMalloc(&q, count * sizeof(T));
    if (e != cudaSuccess) {
        cudaGetLastError();
        return fail(c, WS3D_EMEMORY, "cudaMalloc(%s, %zu bytes): %s", what, count * sizeof(T),
                    cudaGetErrorString(e));
    }
    *p = static_cast<T*>(q);
    c->device_bytes += count * sizeof(T);
    return WS3D_OK;
}

template <class T>
void dfree(ws3d_ctx* c, T*& p, size_t count) {
    if (p) {
        cudaFree(p);
        c->device_bytes -= count * sizeof(T);
        p = nullptr;
    }
}

inline float* owned0(const ws3d_ctx* c, float* base) { return base + c->plane; }
inline size_t owned_elems(const ws3d_ctx* c) { return (size_t)c->nz * c->plane; }

StepParams make_params(const ws3d_ctx* c) {
    StepParams a{};
    a.p = owned0(c, c->buf[c->cur]);
    a.pp = owned0(c, c->buf[c->cur ^ 1]);
    a.c2f = c->c2f ? c->c2f + c->plane : nullptr;
    a.types = c->cells_default ? nullptr : c->types + c->plane;
    a.refl = c->cells_default ? nullptr : c->refl + c->plane;
    a.sponge = c->sponge;
    a.W = c->W;
    a.H = c->H;
    a.pitch = c->pitch;
    a.nz = c->nz;
    a.z0 = c->z0;
    a.Dg = c->Dg;
    a.plane = c->plane;
    a.c2 = c->desc.c_squared;
    a.damping = c->desc.damping;
    a.sponge_w = c->sponge_w;
    return a;
}

// Copy a contiguous host array of nz planes (W x H each) into a pitched slab.
template <class T>
ws3d_status h2d_pitched(ws3d_ctx* c, T* dst_slab, const T* src) {
    cudaError_t e = cudaMemcpy2DAsync(dst_slab + c->plane, c->pitch * sizeof(T), src,
                                      c->W * sizeof(T), c->W * sizeof(T),
                                      (size_t)c->H * c->nz, cudaMemcpyHostToDevice, c->stream);
    if (e != cudaSuccess) return cuda_fail(c, WS3D_EMEMORY, e, "cudaMemcpy2DAsync(h2d)");
    return WS3D_OK;
}

template <class T>
ws3d_status d2h_pitched(ws3d_ctx* c, T* dst, const T* src_slab, ws3d_status code) {
    cudaError_t e = cudaMemcpy2DAsync(dst, c->W * sizeof(T), src_slab + c->plane,
                                      c->pitch * sizeof(T), c->W * sizeof(T),
                                      (size_t)c->H * c->nz, cudaMemcpyDeviceToHost, c->stream);
    if (e != cudaSuccess) return cuda_fail(c, code, e, "cudaMemcpy2DAsync(d2h)");
    return WS3D_OK;
}

// Launch geometry of the z-streaming kernel.
constexpr int kTY = 8;

uint32_t zstream_chunk(const ws3d_ctx* c) {
    const uint32_t tiles = ((c->pitch + 127) / 128) * ((c->H + kTY - 1) / kTY);
    // Enough CTAs for ~8 resident waves over the SMs, but chunks of at least
    // 16 planes so the two extra planes a chunk re-reads stay cheap.
    const uint32_t want = (uint32_t)std::max(1, c->sm_count) * 3u * 8u;
    uint32_t nchunks = std::max(1u, (want + tiles - 1) / tiles);
    uint32_t chunk = (c->nz + nchunks - 1) / nchunks;
    chunk = std::max(chunk, 16u);
    return std::min(chunk, std::max(c->nz, 1u));
}

template <bool kC2F, bool kCells>
void launch_zstream(const ws3d_ctx* c, const StepParams& a) {
    const uint32_t chunk = zstream_chunk(c);
    dim3 block(32, kTY, 1);
    dim3 grid((c->pitch + 127) / 128, (c->H + kTY - 1) / kTY, (c->nz + chunk - 1) / chunk);
    k_step_zstream<kC2F, kCells, kTY><<<grid, block, 0, c->stream>>>(a, chunk);
}

template <bool kC2F, bool kCells>
void launch_naive(const ws3d_ctx* c, const StepParams& a) {
    dim3 block(32, 4, 2);
    dim3 grid((c->W + 31) / 32, (c->H + 3) / 4, (c->nz + 1) / 2);
    k_step_naive<kC2F, kCells><<<grid, block, 0, c->stream>>>(a);
}

ws3d_status ensure_cell_arrays(ws3d_ctx* c);

ws3d_status launch_step(ws3d_ctx* c) {
    StepParams a = make_params(c);
    const bool f = a.c2f != nullptr;
    const bool cells = a.types != nullptr;
    switch (c->desc.variant) {
        case WS3D_VARIANT_NAIVE:
            if (f && cells) launch_naive<true, true>(c, a);
            else if (f) launch_naive<true, false>(c, a);
            else if (cells) launch_naive<false, true>(c, a);
            else launch_naive<false, false>(c, a);
            return check_launch(c, "k_step_naive");
        case WS3D_VARIANT_REFSHAPE: {
            ws3d_status s = ensure_cell_arrays(c);
            if (s != WS3D_OK) return s;
            a.types = c->types + c->plane;
            a.refl = c->refl + c->plane;
            dim3 block(8, 8, 4);
            dim3 grid((c->W + 7) / 8, (c->H + 7) / 8, (c->nz + 3) / 4);
            if (f) k_ref_stencil<true><<<grid, block, 0, c->stream>>>(a);
            else k_ref_stencil<false><<<grid, block, 0, c->stream>>>(a);
            s = check_launch(c, "k_ref_stencil");
            if (s != WS3D_OK) return s;
            const uint64_t n = owned_elems(c);
            k_ref_boundary<<<(unsigned)((n + 255) / 256), 256, 0, c->stream>>>(a.pp, a.types,
                                                                               a.refl, n);
            return check_launch(c, "k_ref_boundary");
        }
        default:
            if (f && cells) launch_zstream<true, true>(c, a);
            else if (f) launch_zstream<true, false>(c, a);
            else if (cells) launch_zstream<false, true>(c, a);
            else launch_zstream<false, false>(c, a);
            return check_launch(c, "k_step_zstream");
    }
}

// Materialise the default face layout as explicit arrays (only the
// reference-shaped comparator reads them).
ws3d_status ensure_cell_arrays(ws3d_ctx* c) {
    if (!c->cells_default || c->types_hold_default) return WS3D_OK;
    if (!c->types) {
        ws3d_status s = dalloc(c, &c->types, c->slab, "cell_types");
        if (s != WS3D_OK) return s;
    }
    if (!c->refl) {
        ws3d_status s = dalloc(c, &c->refl, c->slab, "reflection_coeff");
        if (s != WS3D_OK) return s;
    }
    if (c->cells_default) {
        std::vector<uint8_t> t((size_t)c->W * c->H * c->nz);
        std::vector<float> r(t.size());
        size_t i = 0;
        for (uint32_t zl = 0; zl < c->nz; ++zl) {
            const uint32_t z = c->z0 + zl;
            for (uint32_t y = 0; y < c->H; ++y)
                for (uint32_t x = 0; x < c->W; ++x, ++i) {
                    const bool face = x == 0 || x == c->W - 1 || y == 0 || y == c->H - 1 ||
                                      z == 0 || z == c->Dg - 1;
                    t[i] = face ? kAbsorber : kNormal;
                    r[i] = face ? kFaceReflection : 1.0f;
                }
        }
        WS3D_CUDA(c, cudaMemsetAsync(c->types, 0, c->slab, c->stream), WS3D_EMEMORY);
        WS3D_CUDA(c, cudaMemsetAsync(c->refl, 0, c->slab * sizeof(float), c->stream),
                  WS3D_EMEMORY);
        ws3d_status s = h2d_pitched(c, c->types, t.data());
        if (s == WS3D_OK) s = h2d_pitched(c, c->refl, r.data());
        if (s != WS3D_OK) return s;
        WS3D_CUDA(c, cudaStreamSynchronize(c->stream), WS3D_EMEMORY);
        c->types_hold_default = true;
    }
    return WS3D_OK;
}

bool desc_ok(const ws3d_desc* d, std::string* why) {
    if (!d) { *why = "desc is NULL"; return false; }
    if (d->width == 0 || d->height == 0 || d->depth == 0) { *why = "zero grid dimension"; return false; }
    if (d->width > (1u << 20) || d->height > (1u << 20) || d->depth > (1u << 20)) {
        *why = "grid dimension above 2^20"; return false;
    }
    const uint32_t zb = d->z_begin, ze = d->z_end;
    if (!(zb == 0 && ze == 0) && !(zb < ze && ze <= d->depth)) {
        *why = "z_begin/z_end outside [0, depth]"; return false;
    }
    if (d->variant > WS3D_VARIANT_REFSHAPE) { *why = "unknown variant"; return false; }
    if (d->sponge_width > 4096) { *why = "sponge_width above 4096"; return false; }
    return true;
}

}  // namespace

extern "C" {

uint32_t ws3d_abi_version(void) { return WS3D_ABI_VERSION; }

const char* ws3d_status_string(ws3d_status s) {
    switch (s) {
        case WS3D_OK: return "ok";
        case WS3D_EDEVICE: return "GPU device error";
        case WS3D_ECOMPILE: return "GPU compile error";
        case WS3D_ELAUNCH: return "GPU launch error";
        case WS3D_EMEMORY: return "GPU memory error";
        case WS3D_ESIMULATION: return "simulation error";
        case WS3D_ECOMMAND: return "command error";
        case WS3D_EREADBACK: return "readback error";
        case WS3D_EINVAL: return "invalid argument";
        case WS3D_ETIMEOUT: return "device wait timed out";
        case WS3D_EPEER: return "peer access error";
    }
    return "unknown status";
}

void ws3d_desc_init(ws3d_desc* d, uint32_t width, uint32_t height, uint32_t depth) {
    if (!d) return;
    std::memset(d, 0, sizeof *d);
    d->width = width;
    d->height = height;
    d->depth = depth;
    d->c_squared = 0.25f;
    d->damping = 1.0f;
    d->device = 0;
    d->variant = WS3D_VARIANT_ZSTREAM;
}

ws3d_status ws3d_create(const ws3d_desc* desc, ws3d_ctx** out) {
    if (!out) return WS3D_EINVAL;
    *out = nullptr;
    std::string why;
    if (!desc_ok(desc, &why)) {
        fprintf(stderr, "ws3d_create: %s\n", why.c_str());
        return WS3D_EINVAL;
    }
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) {
        cudaGetLastError();
        fprintf(stderr, "ws3d_create: no CUDA device\n");
        return WS3D_EDEVICE;
    }
    if (desc->device < 0 || desc->device >= ndev) {
        fprintf(stderr, "ws3d_create: device %d out of range (%d devices)\n", desc->device, ndev);
        return WS3D_EDEVICE;
    }
    ws3d_ctx* c = new ws3d_ctx();
    c->desc = *desc;
    c->W = desc->width;
    c->H = desc->height;
    c->Dg = desc->depth;
    c->z0 = (desc->z_end == 0) ? 0 : desc->z_begin;
    c->nz = (desc->z_end == 0) ? desc->depth : desc->z_end - desc->z_begin;
    c->pitch = (c->W + 31u) & ~31u;
    c->plane = (size_t)c->H * c->pitch;
    c->slab = (size_t)(c->nz + 2) * c->plane;

    DeviceGuard g(desc->device);
    auto bail = [&](ws3d_status s) {
        fprintf(stderr, "ws3d_create: %s\n", c->err.c_str());
        ws3d_destroy(c);
        return s;
    };
    if (!g.ok) {
        fail(c, WS3D_EDEVICE, "cudaSetDevice(%d) failed", desc->device);
        return bail(WS3D_EDEVICE);
    }
    cudaDeviceProp prop{};
    cudaError_t e = cudaGetDeviceProperties(&prop, desc->device);
    if (e != cudaSuccess) return bail(cuda_fail(c, WS3D_EDEVICE, e, "cudaGetDeviceProperties"));
    if (prop.major < 10) {
        fail(c, WS3D_ECOMPILE, "device %d is sm_%d%d; this library is built for sm_100a only",
             desc->device, prop.major, prop.minor);
        return bail(WS3D_ECOMPILE);
    }
    c->sm_count = prop.multiProcessorCount;
    e = cudaStreamCreateWithFlags(&c->own_stream, cudaStreamNonBlocking);
    if (e != cudaSuccess) return bail(cuda_fail(c, WS3D_EDEVICE, e, "cudaStreamCreate"));
    c->stream = c->own_stream;

    ws3d_status s;
    for (int b = 0; b < 2; ++b)
        if ((s = dalloc(c, &c->buf[b], c->slab, "pressure")) != WS3D_OK) return bail(s);
    for (int b = 0; b < 2; ++b) {
        e = cudaMemsetAsync(c->buf[b], 0, c->slab * sizeof(float), c->stream);
        if (e != cudaSuccess) return bail(cuda_fail(c, WS3D_EMEMORY, e, "cudaMemsetAsync"));
    }
    if (desc->sponge_width > 0) {
        c->sponge_w = desc->sponge_width;
        std::vector<float> tab(c->sponge_w);
        for (uint32_t d = 0; d < c->sponge_w; ++d) {
            const double t = (double)(c->sponge_w - d) / (double)c->sponge_w;
            tab[d] = (float)(1.0 - (double)desc->sponge_max * t * t);
        }
        if ((s = dalloc(c, &c->sponge, c->sponge_w, "sponge")) != WS3D_OK) return bail(s);
        e = cudaMemcpy(c->sponge, tab.data(), tab.size() * sizeof(float), cudaMemcpyHostToDevice);
        if (e != cudaSuccess) return bail(cuda_fail(c, WS3D_EMEMORY, e, "cudaMemcpy(sponge)"));
    }
    c->red_blocks = (uint32_t)std::max(1, c->sm_count) * 4u;
    if ((s = dalloc(c, &c->red_scratch, (size_t)c->red_blocks + 1, "reduction")) != WS3D_OK)
        return bail(s);
    e = cudaStreamSynchronize(c->stream);
    if (e != cudaSuccess) return bail(cuda_fail(c, WS3D_EDEVICE, e, "cudaStreamSynchronize"));
    *out = c;
    return WS3D_OK;
}

void ws3d_destroy(ws3d_ctx* c) {
    if (!c) return;
    {
        DeviceGuard g(c->desc.device);
        if (c->stream) cudaStreamSynchronize(c->stream);
        for (int b = 0; b < 2; ++b) dfree(c, c->buf[b], c->slab);
        dfree(c, c->c2f, c->slab);
        dfree(c, c->types, c->slab);
        dfree(c, c->refl, c->slab);
        dfree(c, c->sponge, c->sponge_w);
        dfree(c, c->src_off, c->n_src);
        dfree(c, c->wavelet, (size_t)c->n_src * c->wl_len);
        dfree(c, c->red_scratch, (size_t)c->red_blocks + 1);
        if (c->own_stream) cudaStreamDestroy(c->own_stream);
    }
    delete c;
}

const char* ws3d_last_error(const ws3d_ctx* c) { return c ? c->err.c_str() : ""; }

ws3d_status ws3d_upload(ws3d_ctx* c, const float* p, const float* pp) {
    if (!c) return WS3D_EINVAL;
    DeviceGuard g(c->desc.device);
    ws3d_status s = WS3D_OK;
    if (p && (s = h2d_pitched(c, c->buf[c->cur], p)) != WS3D_OK) return s;
    if (pp && (s = h2d_pitched(c, c->buf[c->cur ^ 1], pp)) != WS3D_OK) return s;
    WS3D_CUDA(c, cudaStreamSynchronize(c->stream), WS3D_EMEMORY);
    return WS3D_OK;
}

ws3d_status ws3d_download(ws3d_ctx* c, float* p, float* pp) {
    if (!c || !p) return c ? fail(c, WS3D_EINVAL, "download: pressure is NULL") : WS3D_EINVAL;
    DeviceGuard g(c->desc.device);
    ws3d_status s = d2h_pitched(c, p, c->buf[c->cur], WS3D_EMEMORY);
    if (s == WS3D_OK && pp) s = d2h_pitched(c, pp, c->buf[c->cur ^ 1], WS3D_EMEMORY);
    if (s != WS3D_OK) return s;
    WS3D_CUDA(c, cudaStreamSynchronize(c->stream), WS3D_EMEMORY);
    return WS3D_OK;
}

ws3d_status ws3d_reset(ws3d_ctx* c, const float* p, const float* pp) {
    if (!c) return WS3D_EINVAL;
    c->cur = 0;
    c->step = 0;
    DeviceGuard g(c->desc.device);
    for (int b = 0; b < 2; ++b)
        WS3D_CUDA(c, cudaMemsetAsync(c->buf[b], 0, c->slab * sizeof(float), c->stream),
                  WS3D_EMEMORY);
    return ws3d_upload(c, p, pp);
}

ws3d_status ws3d_set_cells(ws3d_ctx* c, const uint8_t* types, const float* refl) {
    if (!c) return WS3D_EINVAL;
    if ((types == nullptr) != (refl == nullptr))
        return fail(c, WS3D_EINVAL, "set_cells: pass both arrays or neither");
    DeviceGuard g(c->desc.device);
    if (!types) {
        c->cells_default = true;
        return WS3D_OK;
    }
    // Keep the fast path when the arrays equal the default face layout.
    bool same = true;
    size_t i = 0;
    for (uint32_t zl = 0; zl < c->nz && same; ++zl) {
        const uint32_t z = c->z0 + zl;
        for (uint32_t y = 0; y < c->H && same; ++y)
            for (uint32_t x = 0; x < c->W; ++x, ++i) {
                const bool face =
                    x == 0 || x == c->W - 1 || y == 0 || y == c->H - 1 || z == 0 || z == c->Dg - 1;
                const uint8_t t = face ? kAbsorber : kNormal;
                if (types[i] != t || (face && refl[i] != kFaceReflection)) {
                    same = false;
                    break;
                }
            }
    }
    if (same) {
        c->cells_default = true;
        return WS3D_OK;
    }
    for (size_t k = 0, n = (size_t)c->W * c->H * c->nz; k < n; ++k)
        if (types[k] > kObstacle)
            return fail(c, WS3D_EINVAL, "set_cells: cell type %u at index %zu is not 0..3",
                        (unsigned)types[k], k);
    ws3d_status s;
    if (!c->types && (s = dalloc(c, &c->types, c->slab, "cell_types")) != WS3D_OK) return s;
    if (!c->refl && (s = dalloc(c, &c->refl, c->slab, "reflection_coeff")) != WS3D_OK) return s;
    WS3D_CUDA(c, cudaMemsetAsync(c->types, 0, c->slab, c->stream), WS3D_EMEMORY);
    WS3D_CUDA(c, cudaMemsetAsync(c->refl, 0, c->slab * sizeof(float), c->stream), WS3D_EMEMORY);
    if ((s = h2d_pitched(c, c->types, types)) != WS3D_OK) return s;
    if ((s = h2d_pitched(c, c->refl, refl)) != WS3D_OK) return s;
    WS3D_CUDA(c, cudaStreamSynchronize(c->stream), WS3D_EMEMORY);
    c->cells_default = false;
    c->types_hold_default = false;
    return WS3D_OK;
}

ws3d_status ws3d_set_c2_field(ws3d_ctx* c, const float* c2) {
    if (!c) return WS3D_EINVAL;
    DeviceGuard g(c->desc.device);
    if (!c2) {
        dfree(c, c->c2f, c->slab);
        return WS3D_OK;
    }
    ws3d_status s;
    if (!c->c2f) {
        if ((s = dalloc(c, &c->c2f, c->slab, "c2_field")) != WS3D_OK) return s;
        WS3D_CUDA(c, cudaMemsetAsync(c->c2f, 0, c->slab * sizeof(float), c->stream),
                  WS3D_EMEMORY);
    }
    if ((s = h2d_pitched(c, c->c2f, c2)) != WS3D_OK) return s;
    WS3D_CUDA(c, cudaStreamSynchronize(c->stream), WS3D_EMEMORY);
    return WS3D_OK;
}

ws3d_status ws3d_set_sources(ws3d_ctx* c, uint32_t n, const uint32_t* xyz, const float* wavelet,
                             uint64_t len) {
    if (!c) return WS3D_EINVAL;
    if (n > 0 && (!xyz || !wavelet || len == 0))
        return fail(c, WS3D_EINVAL, "set_sources: xyz/wavelet missing");
    if (n > 65536) return fail(c, WS3D_EINVAL, "set_sources: more than 65536 sources");
    DeviceGuard g(c->desc.device);
    WS3D_CUDA(c, cudaStreamSynchronize(c->stream), WS3D_EDEVICE);
    dfree(c, c->src_off, c->n_src);
    dfree(c, c->wavelet, (size_t)c->n_src * c->wl_len);
    c->n_src = 0;
    c->wl_len = 0;
    // Keep only the sources inside the owned planes, in their given order.
    std::vector<uint64_t> off;
    std::vector<float> wl;
    for (uint32_t k = 0; k < n; ++k) {
        const uint32_t x = xyz[3 * k], y = xyz[3 * k + 1], z = xyz[3 * k + 2];
        if (x >= c->W || y >= c->H || z >= c->Dg)
            return fail(c, WS3D_EINVAL, "set_sources: source %u at (%u,%u,%u) outside the grid",
                        k, x, y, z);
        if (z < c->z0 || z >= c->z0 + c->nz) continue;
        off.push_back((uint64_t)(z - c->z0 + 1) * c->plane + (uint64_t)y * c->pitch + x);
        wl.insert(wl.end(), wavelet + (size_t)k * len, wavelet + (size_t)(k + 1) * len);
    }
    if (off.empty()) return WS3D_OK;
    ws3d_status s;
    if ((s = dalloc(c, &c->src_off, off.size(), "sources")) != WS3D_OK) return s;
    if ((s = dalloc(c, &c->wavelet, wl.size(), "wavelet")) != WS3D_OK) return s;
    WS3D_CUDA(c, cudaMemcpy(c->src_off, off.data(), off.size() * 8, cudaMemcpyHostToDevice),
              WS3D_EMEMORY);
    WS3D_CUDA(c, cudaMemcpy(c->wavelet, wl.data(), wl.size() * 4, cudaMemcpyHostToDevice),
              WS3D_EMEMORY);
    c->n_src = (uint32_t)off.size();
    c->wl_len = len;
    return WS3D_OK;
}

ws3d_status ws3d_step(ws3d_ctx* c, uint64_t n) {
    if (!c) return WS3D_EINVAL;
    DeviceGuard g(c->desc.device);
    for (uint64_t i = 0; i < n; ++i) {
        if (c->n_src) {
            k_inject_sources<<<1, 32, 0, c->stream>>>(c->buf[c->cur], c->buf[c->cur ^ 1],
                                                      c->src_off, c->wavelet, c->n_src,
                                                      c->wl_len, c->step);
            ws3d_status s = check_launch(c, "k_inject_sources");
            if (s != WS3D_OK) return s;
        }
        ws3d_status s = launch_step(c);
        if (s != WS3D_OK) return s;
        c->cur ^= 1;
        c->step++;
    }
    return WS3D_OK;
}

ws3d_status ws3d_inject_impulse(ws3d_ctx* c, uint32_t x, uint32_t y, uint32_t z, float amp) {
    if (!c) return WS3D_EINVAL;
    if (x >= c->W || y >= c->H || z >= c->Dg) return WS3D_OK;  // grid3d.rs:147
    if (z < c->z0 || z >= c->z0 + c->nz) return WS3D_OK;      // another slab owns it
    DeviceGuard g(c->desc.device);
    const uint64_t off = (uint64_t)(z - c->z0 + 1) * c->plane + (uint64_t)y * c->pitch + x;
    k_inject_point<<<1, 32, 0, c->stream>>>(c->buf[c->cur], c->buf[c->cur ^ 1], off, amp);
    return check_launch(c, "k_inject_point");
}

ws3d_status ws3d_inject_spherical_impulse(ws3d_ctx* c, uint32_t cx, uint32_t cy, uint32_t cz,
                                          float amp, float radius) {
    if (!c) return WS3D_EINVAL;
    if (!(radius >= 0.0f) || radius > 1024.0f)
        return fail(c, WS3D_EINVAL, "inject_spherical_impulse: radius %g outside [0, 1024]",
                    (double)radius);
    DeviceGuard g(c->desc.device);
    const int r = (int)radius;
    const float r_sq = radius * radius;
    std::vector<uint64_t> off;
    std::vector<float> fac;
    for (int dz = -r; dz <= r; ++dz)
        for (int dy = -r; dy <= r; ++dy)
            for (int dx = -r; dx <= r; ++dx) {
                const long long x = (long long)cx + dx, y = (long long)cy + dy,
                                z = (long long)cz + dz;
                if (x < 0 || y < 0 || z < 0 || x >= c->W || y >= c->H || z >= c->Dg) continue;
                const float dist_sq = (float)(dx * dx + dy * dy + dz * dz);
                if (!(dist_sq <= r_sq)) continue;
                if (z < c->z0 || z >= (long long)c->z0 + c->nz) continue;
                off.push_back((uint64_t)(z - c->z0 + 1) * c->plane + (uint64_t)y * c->pitch +
                              (uint64_t)x);
                fac.push_back(expf(-dist_sq / (2.0f * radius)));
            }
    if (off.empty()) return WS3D_OK;
    uint64_t* d_off = nullptr;
    float* d_fac = nullptr;
    ws3d_status s;
    if ((s = dalloc(c, &d_off, off.size(), "impulse offsets")) != WS3D_OK) return s;
    if ((s = dalloc(c, &d_fac, fac.size(), "impulse factors")) != WS3D_OK) {
        dfree(c, d_off, off.size());
        return s;
    }
    cudaError_t e1 = cudaMemcpyAsync(d_off, off.data(), off.size() * 8, cudaMemcpyHostToDevice,
                                     c->stream);
    cudaError_t e2 = cudaMemcpyAsync(d_fac, fac.data(), fac.size() * 4, cudaMemcpyHostToDevice,
                                     c->stream);
    if (e1 == cudaSuccess && e2 == cudaSuccess) {
        const uint32_t n = (uint32_t)off.size();
        k_inject_table<<<(n + 255) / 256, 256, 0, c->stream>>>(c->buf[c->cur], c->buf[c->cur ^ 1],
                                                              d_off, d_fac, n, amp);
        s = check_launch(c, "k_inject_table");
    } else {
        s = cuda_fail(c, WS3D_EMEMORY, e1 != cudaSuccess ? e1 : e2, "cudaMemcpyAsync(impulse)");
    }
    cudaStreamSynchronize(c->stream);
    dfree(c, d_off, off.size());
    dfree(c, d_fac, fac.size());
    return s;
}

ws3d_status ws3d_energy(ws3d_ctx* c, double* out) {
    if (!c || !out) return WS3D_EINVAL;
    DeviceGuard g(c->desc.device);
    const uint64_t rows = (uint64_t)c->nz * c->H;
    k_energy_partials<<<c->red_blocks, kRedThreads, 0, c->stream>>>(
        owned0(c, c->buf[c->cur]), c->W, c->pitch, rows, c->red_scratch);
    ws3d_status s = check_launch(c, "k_energy_partials");
    if (s != WS3D_OK) return s;
    k_fold_partials<<<1, kRedThreads, 0, c->stream>>>(c->red_scratch, c->red_blocks,
                                                      c->red_scratch + c->red_blocks);
    if ((s = check_launch(c, "k_fold_partials")) != WS3D_OK) return s;
    WS3D_CUDA(c, cudaMemcpyAsync(out, c->red_scratch + c->red_blocks, sizeof(double),
                                 cudaMemcpyDeviceToHost, c->stream),
              WS3D_EREADBACK);
    WS3D_CUDA(c, cudaStreamSynchronize(c->stream), WS3D_EREADBACK);
    return WS3D_OK;
}

ws3d_status ws3d_max_pressure(ws3d_ctx* c, float* out) {
    if (!c || !out) return WS3D_EINVAL;
    DeviceGuard g(c->desc.device);
    const uint64_t rows = (uint64_t)c->nz * c->H;
    float* part = reinterpret_cast<float*>(c->red_scratch);
    k_maxabs_partials<<<c->red_blocks, kRedThreads, 0, c->stream>>>(
        owned0(c, c->buf[c->cur]), c->W, c->pitch, rows, part);
    ws3d_status s = check_launch(c, "k_maxabs_partials");
    if (s != WS3D_OK) return s;
    float* res = reinterpret_cast<float*>(c->red_scratch + c->red_blocks);
    k_fold_max<<<1, kRedThreads, 0, c->stream>>>(part, c->red_blocks, res);
    if ((s = check_launch(c, "k_fold_max")) != WS3D_OK) return s;
    WS3D_CUDA(c, cudaMemcpyAsync(out, res, sizeof(float), cudaMemcpyDeviceToHost, c->stream),
              WS3D_EREADBACK);
    WS3D_CUDA(c, cudaStreamSynchronize(c->stream), WS3D_EREADBACK);
    return WS3D_OK;
}

size_t ws3d_memory_usage(const ws3d_ctx* c) { return c ? c->device_bytes : 0; }

ws3d_status ws3d_sync(ws3d_ctx* c) {
    if (!c) return WS3D_EINVAL;
    DeviceGuard g(c->desc.device);
    WS3D_CUDA(c, cudaStreamSynchronize(c->stream), WS3D_ELAUNCH);
    return WS3D_OK;
}

ws3d_status ws3d_set_stream(ws3d_ctx* c, void* stream) {
    if (!c) return WS3D_EINVAL;
    DeviceGuard g(c->desc.device);
    WS3D_CUDA(c, cudaStreamSynchronize(c->stream), WS3D_EDEVICE);
    c->stream = stream ? static_cast<cudaStream_t>(stream) : c->own_stream;
    return WS3D_OK;
}

ws3d_status ws3d_get_stream(const ws3d_ctx* c, void** stream) {
    if (!c || !stream) return WS3D_EINVAL;
    *stream = c->stream;
    return WS3D_OK;
}

ws3d_status ws3d_stats_get(const ws3d_ctx* c, ws3d_stats* o) {
    if (!c || !o) return WS3D_EINVAL;
    std::memset(o, 0, sizeof *o);
    o->step = c->step;
    o->kernel_launches = c->launches;
    o->device_bytes = c->device_bytes;
    o->width = c->W;
    o->height = c->H;
    o->depth = c->Dg;
    o->z_begin = c->z0;
    o->z_end = c->z0 + c->nz;
    o->pitch = c->pitch;
    o->variant = c->desc.variant;
    o->has_c2_field = c->c2f != nullptr;
    o->has_cell_field = !c->cells_default;
    o->n_sources = c->n_src;
    return WS3D_OK;
}

}  // extern "C"
