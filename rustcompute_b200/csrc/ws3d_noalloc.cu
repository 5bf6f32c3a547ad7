// ws3d_noalloc.cu -- field energy without any device allocation.
//
// ws3d_energy() reduces through a scratch buffer that ws3d_create() obtained
// with cudaMalloc.  Some callers cannot allocate device memory at the point
// where they want this number: a real-time loop such as an audio callback
// that must never block on the device synchronisation cudaMalloc/cudaFree
// can imply, or a host application that owns every byte of device memory
// through its own pool and forbids libraries from allocating.  For them,
// ws3d_field_energy_static() reduces a caller-owned device field into a
// caller-owned device result and keeps its scratch in the fixed array below,
// which every GPU that loads this library holds until the process exits.
//
// The array's device address is looked up once per device and cached; a
// cudaDeviceReset() of that device destroys the module that holds it, so
// calls after such a reset are not supported (the rest of the library's
// device state does not survive a reset either).
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
// Each warp walks whole rows (warp w takes rows w, w + 16, ...), its lanes
// stride along the row: coalesced, and no per-element index division.
__global__ void __launch_bounds__(kThreads) k_plane_energy(const float* __restrict__ field,
                                                           uint32_t W, uint32_t H,
                                                           uint32_t pitch, double* partials) {
    const uint32_t z = blockIdx.x;
    const float* plane = field + (size_t)z * H * pitch;
    double acc = 0.0;
    const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
    for (uint32_t y = warp; y < H; y += kThreads / 32) {
        const float* row = plane + (size_t)y * pitch;
        for (uint32_t x = lane; x < W; x += 32) {
            const float v = row[x];
            acc += (double)v * (double)v;
        }
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
    // An error the caller's own earlier work left pending is reported, not
    // consumed: it stays pending for the caller, and nothing is launched.
    cudaError_t e = cudaPeekAtLastError();
    if (e != cudaSuccess)
        return report(errbuf, errlen, WS3D_ELAUNCH,
                      "field_energy_static: a CUDA error was already pending before this call "
                      "(%s); nothing was launched", cudaGetErrorString(e));
    int dev = -1;
    e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices)
        return report(errbuf, errlen, WS3D_EDEVICE, "field_energy_static: no current device (%s)",
                      cudaGetErrorString(e));
    double* partials = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_setup_mutex);
        if (!g_partials_addr[dev]) {
            // First call on this device: resolve the array's device address
            // with the device current.  This set-up belongs before any stream
            // capture: make the first call on each device outside one.
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
