// ws3d_noalloc.cu -- field energy without any device allocation.
//
// ws3d_energy() reduces through a scratch buffer that ws3d_create() obtained
// with cudaMalloc.  Some callers cannot allocate device memory at the point
// where they want this number: code being recorded into a CUDA graph (stream
// capture rejects cudaMalloc/cudaFree), a real-time loop such as an audio
// callback that must never block on the implicit device synchronisation of
// cudaMalloc/cudaFree, or a host application that owns every byte of device
// memory through its own pool and forbids libraries from allocating.  For
// them, ws3d_field_energy_static() reduces a caller-owned device field into a
// caller-owned device result and keeps its scratch in the fixed array below,
// which every GPU that loads this library holds until the process exits.
#include "ws3d.h"

#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

namespace {

// One partial sum per z-plane: 8192 doubles = 64 KiB per device.
static __device__ __align__(256) double g_plane_partials[WS3D_STATIC_ENERGY_MAX_PLANES];

constexpr int kThreads = 512;
constexpr int kMaxDevices = 64;

// Host-side copies of the array's device address, one per device.  In host
// code `g_plane_partials` only names a host stand-in, never the device
// memory, so the address is looked up once per device with that device
// current and cached here.
double* g_partials_addr[kMaxDevices] = {};
std::mutex g_setup_mutex;

__device__ __forceinline__ double warp_sum(double v) {
    for (int o = 16; o > 0; o >>= 1) v += __shfl_down_sync(0xffffffffu, v, o);
    return v;
}

__device__ double block_sum(double v) {
    __shared__ double sm[kThreads / 32];
    v = warp_sum(v);
    if ((threadIdx.x & 31) == 0) sm[threadIdx.x >> 5] = v;
    __syncthreads();
    double t = 0.0;
    if (threadIdx.x < 32) {
        t = threadIdx.x < kThreads / 32 ? sm[threadIdx.x] : 0.0;
        t = warp_sum(t);
    }
    return t;  // valid in thread 0
}

// Block z sums p^2 over plane z (W x H cells, row pitch `pitch` floats) and
// writes partials[z]; every partial the fold reads is written by this launch.
__global__ void __launch_bounds__(kThreads) k_plane_energy(const float* __restrict__ field,
                                                           uint32_t W, uint32_t H,
                                                           uint32_t pitch, double* partials) {
    const uint32_t z = blockIdx.x;
    const float* plane = field + (size_t)z * H * pitch;
    double acc = 0.0;
    const uint64_t n = (uint64_t)W * H;
    for (uint64_t i = threadIdx.x; i < n; i += kThreads) {
        const uint64_t y = i / W, x = i - y * W;
        const float v = plane[y * pitch + x];
        acc += (double)v * (double)v;
    }
    acc = block_sum(acc);
    if (threadIdx.x == 0) partials[z] = acc;
}

// Fold partials[0..nz) in a fixed order into *result (deterministic).
__global__ void __launch_bounds__(kThreads) k_fold_planes(const double* partials, uint32_t nz,
                                                          double* result) {
    double acc = 0.0;
    for (uint32_t i = threadIdx.x; i < nz; i += kThreads) acc += partials[i];
    acc = block_sum(acc);
    if (threadIdx.x == 0) *result = acc;
}

ws3d_status report(char* errbuf, size_t errlen, ws3d_status s, const char* fmt, ...) {
    if (errbuf && errlen) {
        va_list ap;
        va_start(ap, fmt);
        vsnprintf(errbuf, errlen, fmt, ap);
        va_end(ap);
    }
    return s;
}

}  // namespace

extern "C" ws3d_status ws3d_field_energy_static(const float* field, uint32_t width,
                                                uint32_t height, uint32_t nz, uint32_t pitch,
                                                double* result, void* stream, char* errbuf,
                                                size_t errlen) {
    if (errbuf && errlen) errbuf[0] = '\0';
    if (!field || !result)
        return report(errbuf, errlen, WS3D_EINVAL, "field_energy_static: NULL field or result");
    if (nz > WS3D_STATIC_ENERGY_MAX_PLANES)
        return report(errbuf, errlen, WS3D_EINVAL,
                      "field_energy_static: %u planes exceed the fixed scratch of %u planes",
                      nz, (unsigned)WS3D_STATIC_ENERGY_MAX_PLANES);
    if (pitch < width)
        return report(errbuf, errlen, WS3D_EINVAL,
                      "field_energy_static: pitch %u is smaller than width %u", pitch, width);
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices)
        return report(errbuf, errlen, WS3D_EDEVICE, "field_energy_static: no current device (%s)",
                      cudaGetErrorString(e));
    double* partials = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_setup_mutex);
        if (!g_partials_addr[dev]) {
            // First call on this device: resolve the array's device address
            // with the device current.  Not capturable: make this first call
            // outside any stream capture.
            void* addr = nullptr;
            e = cudaGetSymbolAddress(&addr, g_plane_partials);
            if (e != cudaSuccess || !addr)
                return report(errbuf, errlen, WS3D_EDEVICE,
                              "field_energy_static: cudaGetSymbolAddress failed on device %d: %s",
                              dev, cudaGetErrorString(e));
            g_partials_addr[dev] = static_cast<double*>(addr);
        }
        partials = g_partials_addr[dev];
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (nz > 0) {
        k_plane_energy<<<nz, kThreads, 0, s>>>(field, width, height, pitch, partials);
        e = cudaGetLastError();
        if (e != cudaSuccess)
            return report(errbuf, errlen, WS3D_ELAUNCH, "field_energy_static: %s",
                          cudaGetErrorString(e));
    }
    k_fold_planes<<<1, kThreads, 0, s>>>(partials, nz, result);
    e = cudaGetLastError();
    if (e != cudaSuccess)
        return report(errbuf, errlen, WS3D_ELAUNCH, "field_energy_static: %s",
                      cudaGetErrorString(e));
    return WS3D_OK;
}
