// ws3d_api.cu -- host side of libws3d.so: the C-ABI declared in include/ws3d.h.
//
// The context mirrors GpuBackend3D (crates/ringkernel-wavesim3d/src/simulation/
// gpu_backend.rs:172-494): it owns the device fields, launches the step and
// keeps the buffer roles (pressure / pressure_prev) by swapping indices
// instead of copying, exactly like gpu_backend.rs:372.
#include "ws3d.h"
#include "ws3d_kernels.cuh"
#include "ws3d_nvtx.h"
#include "ws3d_async.cuh"
#include "ws3d_persistent.cuh"
#include "ws3d_smemstep.cuh"
#include "ws3d_tb.cuh"
#include "ws3d_tma.cuh"
#include "ws3d_volume.cuh"

#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <atomic>
#include <chrono>
#include <thread>
#include <vector>

using namespace ws3d;

struct ws3d_ctx {
    ws3d_desc desc{};
    uint32_t W = 0, H = 0, Dg = 0, z0 = 0, nz = 0, pitch = 0;
    size_t plane = 0;       // H * pitch floats
    size_t slab = 0;        // (nz + 2) * plane floats (ghost below + owned + ghost above)
    // Field buffers: buf[ip] = pressure, buf[ipp] = pressure_prev.  Buffers 2
    // and 3 are allocated on first use of the two-step (temporally blocked)
    // pass, which writes both new fields into free buffers.  buf[b] points at
    // ghost plane -1; a z-slab's field buffers hold gd = 2 ghost planes per
    // side (allocation base buf[b] - plane), one GPU's gd = 1.
    float* buf[4] = {nullptr, nullptr, nullptr, nullptr};
    uint32_t gd = 1;
    int ip = 0, ipp = 1;
    float* c2f = nullptr;   // slab-shaped, or nullptr
    uint8_t* types = nullptr;
    float* refl = nullptr;
    bool cells_default = true;     // kernels evaluate the default face layout analytically
    bool types_hold_default = false;  // types/refl arrays currently hold that default layout
    float* sponge = nullptr;
    uint32_t sponge_w = 0;
    bool sponge_monotone = true;   // table non-decreasing and <= 1 (the lean cell rule's premise)
    uint64_t* src_off = nullptr;
    float* wavelet = nullptr;
    uint32_t n_src = 0;
    uint64_t wl_len = 0;
    long long* src_ghost = nullptr;   // per source: offsets in the lower / upper neighbour's copy, or -1
    std::vector<uint32_t> src_xyz;    // local sources, global coordinates
    // the whole source list as given (all slabs get the same one): two-step
    // launches on z-slabs also apply the sources of the ghost planes
    std::vector<uint32_t> gsrc_xyz;
    std::vector<float> gsrc_wl;
    uint32_t n_src_global = 0;
    uint64_t* tb_src_off = nullptr;   // z-slab two-step table: sources on planes -1 .. nz
    float* tb_wavelet = nullptr;
    uint32_t tb_n_src = 0;
    double* red_scratch = nullptr;  // reduction partials + result
    uint32_t red_blocks = 0;
    cudaStream_t own_stream = nullptr;
    cudaStream_t stream = nullptr;
    uint64_t step = 0;
    uint64_t launches = 0;
    size_t device_bytes = 0;
    int sm_count = 0;
    std::string err;

    // z-slab halo exchange
    bool halo = false;               // neighbours attached
    bool host_ordered = false;       // same-device neighbours: stream order, no device waits
    bool halo_synced = false;        // ghost planes hold the neighbours' current boundary planes
    // neighbours' field buffers (mapped; their plane -1), permuted together
    // with buf[] so that index k is the neighbour's buffer in the same role
    float* lo_base[4] = {nullptr, nullptr, nullptr, nullptr};
    float* hi_base[4] = {nullptr, nullptr, nullptr, nullptr};
    const float* lo_c2 = nullptr;    // neighbours' c2 fields (plane -1), or null
    const float* hi_c2 = nullptr;
    uint32_t lo_caps = 0, hi_caps = 0;   // WS3D_HALO_CAP_* of the neighbours
    uint32_t lo_nz = 0, hi_nz = 0;       // their owned planes
    float lo_c2u = 0.f, hi_c2u = 0.f;    // their uniform c2
    uint64_t lo_ghost_off = 0;       // elements from lower's buffer base to its upper ghost
    uint32_t hdepth = 1;             // steps per exchange (ws3d_halo_set_depth)
    bool deep_ok = false;            // neighbours' copies of our two edge planes are current
    unsigned long long* flags = nullptr;     // [0] from lower, [1] from upper, [2] status
    unsigned long long* lo_flag = nullptr;   // lower neighbour's flags[1]
    unsigned long long* hi_flag = nullptr;   // upper neighbour's flags[0]
    std::vector<void*> ipc_opened;   // mappings to close on destroy
    uint64_t halo_steps = 0;         // steps since the last halo sync
    uint64_t budget_ns = 2000000000ull;

    // optional per-launch timing of the step kernel (ws3d_step_timed): a ring
    // of kTimedRing event pairs; tev_rec launches recorded, the first
    // tev_done of them already summed into tev_ms
    std::vector<cudaEvent_t> tev;
    uint64_t tev_rec = 0, tev_done = 0;
    double tev_ms = 0.0;

    // TMA kernels: tensor maps of every field buffer in every role and of c2
    // (index = buffer; permuted together with buf[] after a two-step launch)
    CUtensorMap mapP[4];   // one step, pressure role: box 136 x (TY+2) x 1
    CUtensorMap mapT[4];   // one step, p_prev role:   box 128 x TY x 1
    CUtensorMap mapC2;     // one step, c2:            box 128 x TY x 1
    CUtensorMap mapA[4];   // two steps, pressure role: box 136 x (TY+4) x 1
    CUtensorMap mapB[4];   // two steps, p_prev role:   box 136 x (TY+2) x 1
    CUtensorMap mapC2b;    // two steps, c2:            box 136 x (TY+2) x 1
    // z-slabs at temporal depth 2: the neighbours' field buffers (index as
    // lo_base / hi_base, permuted with them) and c2 fields in the p_prev role,
    // over their planes -1 .. nz: the two-step kernel stages their edge planes
    // of p_{t-1} and c2 from these (plain TMA loads of peer memory)
    CUtensorMap mapBlo[4], mapBhi[4], mapC2lo, mapC2hi;
    bool peer_maps = false;
    bool tma_maps = false, tma_c2_map = false;
    bool tb_buffers = false;   // buffers 2 and 3 allocated, their maps encoded
    bool tb_failed = false;    // their allocation failed: run single steps
    int tma_grid[4] = {0, 0, 0, 0};  // co-resident CTAs: [c2 field + 2 * lean rule]
    int tb_grid[8] = {0, 0, 0, 0, 0, 0, 0, 0};  // [c2 field + 2 * slab + 4 * deep pipeline]
    int tb_stages_env = 0;  // WS3D_TWO_STEP_STAGES read at create; 0: by plane width
    uint64_t tb_launches = 0;
    int async_grid[2] = {0, 0};
    uint32_t tma_min_chunk = 32;  // WS3D_TMA_MIN_CHUNK (schedule tuning), read at create
    // persistent launches of small one-GPU grids keep the field in shared
    // memory (k_persistent_smem); WS3D_PERSISTENT_SMEM=0 at create turns it off
    bool smem_persistent = true;
    // its block shape per c2 instance, found on first use: 0 unknown, 1 fits, -1 does not
    int smem_plan[2] = {0, 0};
    uint32_t smem_by[2] = {0, 0}, smem_bz[2] = {0, 0};
    // its face exchange rows (tagged words) and the next launch's first tag
    unsigned long long* smem_xch = nullptr;
    size_t smem_xch_words = 0;
    uint32_t smem_tag = 0;

    // persistent mode: co-resident CTAs of k_persistent per instantiation
    int pers_resident[4] = {0, 0, 0, 0};
    uint64_t persistent_launches = 0;

    // resident (command-driven) mode: queues and control block in mapped
    // host memory; see ws3d_resident_* and k_resident
    bool res_active = false;       // started and not shut down
    bool res_alive = false;        // a launch is (or may still be) on the GPU
    bool res_terminated = false;   // the kernel left after TERMINATE
    void* res_mem = nullptr;       // cudaHostAlloc'd block (host view; mapped)
    size_t res_bytes = 0;
    ResidentCtrl* res_ctrl = nullptr;
    ResQueue* res_h2k = nullptr;
    ResMsg* res_h2k_slots = nullptr;
    ResQueue* res_k2h = nullptr;
    ResMsg* res_k2h_slots = nullptr;
    uint64_t res_h2k_tail = 0;     // host producer index
    uint64_t res_k2h_head = 0;     // host consumer index
    ws3d_resident_config res_cfg{};
    cudaEvent_t res_done = nullptr;
    cudaStream_t res_side = nullptr;  // downloads while the kernel stays resident
    uint64_t res_launches = 0;
    int res_role[2] = {0, 1};      // field buffers of roles 0 / 1 of the current launch
    uint64_t res_step0 = 0;        // step count at the current launch
    int res_resident = 0;          // co-resident CTAs of k_resident

    // volume rendering: normalised f16 copy of the field and the image
    __half* vol16 = nullptr;
    size_t vol_elems = 0;
    float4* img = nullptr;
    size_t img_elems = 0;
};

namespace {

constexpr size_t kFlagWords = 32;
// Flag block words: 0 / 1 the lower / upper neighbour's flag, 2 status, 4 the
// persistent grid barrier's arrival counter, 6 the resident kernel's decision,
// 8 / 9 the neighbour-wait accumulators (ns, count).
constexpr size_t kBarWord = 4;
constexpr size_t kWaitAccWord = 8;

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

// Calls that use the context's stream or its fields are refused while a
// resident kernel owns them (ws3d_resident_shutdown hands them back).
#define WS3D_NOT_RESIDENT(ctx)                                                        \
    do {                                                                              \
        if ((ctx) && (ctx)->res_active)                                               \
            return fail(ctx, WS3D_ECOMMAND,                                           \
                        "%s: a resident kernel owns this context; use ws3d_resident_* " \
                        "or ws3d_resident_shutdown first", __func__);                 \
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

// Field buffer b: one allocation of nz + 2 * gd planes, buf[b] at plane -1.
inline size_t fbuf_elems(const ws3d_ctx* c) { return (size_t)(c->nz + 2 * c->gd) * c->plane; }
inline float* fbuf_base(const ws3d_ctx* c, int b) {
    return c->buf[b] ? c->buf[b] - (size_t)(c->gd - 1) * c->plane : nullptr;
}
ws3d_status falloc(ws3d_ctx* c, int b, const char* what) {
    float* q = nullptr;
    ws3d_status s = dalloc(c, &q, fbuf_elems(c), what);
    if (s != WS3D_OK) return s;
    c->buf[b] = q + (size_t)(c->gd - 1) * c->plane;
    cudaError_t e = cudaMemsetAsync(q, 0, fbuf_elems(c) * sizeof(float), c->stream);
    if (e != cudaSuccess) return cuda_fail(c, WS3D_EMEMORY, e, "cudaMemsetAsync(field)");
    return WS3D_OK;
}
void ffree(ws3d_ctx* c, int b) {
    float* q = fbuf_base(c, b);
    dfree(c, q, fbuf_elems(c));
    c->buf[b] = nullptr;
}

StepParams make_params(const ws3d_ctx* c) {
    StepParams a{};
    a.p = owned0(c, c->buf[c->ip]);
    a.pp = owned0(c, c->buf[c->ipp]);
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
    if (c->halo) {
        const int nxt = c->ipp;   // the neighbour's buffer in the same role
        a.peer_lo = c->lo_base[nxt] ? c->lo_base[nxt] + c->lo_ghost_off : nullptr;
        a.peer_hi = c->hi_base[nxt];
        if (c->hdepth == 2) {  // the neighbours' second ghost planes too
            a.peer_lo2 = a.peer_lo ? a.peer_lo + c->plane : nullptr;
            a.peer_hi2 = a.peer_hi ? a.peer_hi - c->plane : nullptr;
        }
        if (!c->host_ordered) {
            a.wait_lo = c->lo_base[0] ? c->flags + 0 : nullptr;
            a.wait_hi = c->hi_base[0] ? c->flags + 1 : nullptr;
        }
        // Before step s a neighbour raises its flag to s+1 (after its step s-1
        // and after its sources of step s reached our ghost planes).
        a.wait_val = c->halo_steps + 1;
    }
    // bound of every device-side wait: neighbour flags and the grid barriers
    // of the persistent and resident kernels (one GPU too)
    a.budget_ns = c->budget_ns;
    a.status = reinterpret_cast<unsigned int*>(c->flags + 2);
    a.wait_acc = c->flags + kWaitAccWord;
    return a;
}

// Copy a contiguous host array of nz planes (W x H each) into a pitched slab
// (one linear copy when rows carry no padding, W a multiple of 32).
template <class T>
ws3d_status h2d_pitched(ws3d_ctx* c, T* dst_slab, const T* src) {
    const size_t rows = (size_t)c->H * c->nz;
    cudaError_t e =
        c->pitch == c->W
            ? cudaMemcpyAsync(dst_slab + c->plane, src, rows * c->W * sizeof(T),
                              cudaMemcpyHostToDevice, c->stream)
            : cudaMemcpy2DAsync(dst_slab + c->plane, c->pitch * sizeof(T), src, c->W * sizeof(T),
                                c->W * sizeof(T), rows, cudaMemcpyHostToDevice, c->stream);
    if (e != cudaSuccess) return cuda_fail(c, WS3D_EMEMORY, e, "cudaMemcpyAsync(h2d)");
    return WS3D_OK;
}

template <class T>
ws3d_status d2h_pitched(ws3d_ctx* c, T* dst, const T* src_slab, ws3d_status code) {
    const size_t rows = (size_t)c->H * c->nz;
    cudaError_t e =
        c->pitch == c->W
            ? cudaMemcpyAsync(dst, src_slab + c->plane, rows * c->W * sizeof(T),
                              cudaMemcpyDeviceToHost, c->stream)
            : cudaMemcpy2DAsync(dst, c->W * sizeof(T), src_slab + c->plane, c->pitch * sizeof(T),
                                c->W * sizeof(T), rows, cudaMemcpyDeviceToHost, c->stream);
    if (e != cudaSuccess) return cuda_fail(c, code, e, "cudaMemcpyAsync(d2h)");
    return WS3D_OK;
}

// Halo flag block: [0] raised by the lower neighbour, [1] by the upper one,
// [2] status word; padded to 256 bytes.


// Launch geometry of the z-streaming kernel (ws3d_index.h).
constexpr int kTY = 8;

template <bool kC2F, bool kCells>
void launch_zstream(const ws3d_ctx* c, const StepParams& a) {
    const uint32_t chunk = zs_zchunk<kTY>(c->pitch, c->H, c->nz, c->sm_count);
    uint32_t gx, gy, gz;
    zs_grid<kTY>(c->pitch, c->H, c->nz, chunk, &gx, &gy, &gz);
    k_step_zstream<kC2F, kCells, kTY><<<dim3(gx, gy, gz), dim3(32, kTY, 1), 0, c->stream>>>(a, chunk);
}

// ---- TMA kernel (single GPU, default face layout) --------------------------
constexpr int kTmaTY = 8;

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000,
                                             cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
        else
            cudaGetLastError();
    });
    return fn;
}

// 3-D map over a slab-shaped buffer: dims {pitch, H, planes} (default nz+2
// from ghost plane -1), fp32, zero fill.
bool encode_slab_map(const ws3d_ctx* c, CUtensorMap* m, const float* base, uint32_t box_x,
                     uint32_t box_y, uint64_t planes = 0) {
    PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
    if (!enc) return false;
    const cuuint64_t dims[3] = {c->pitch, c->H, planes ? planes : (cuuint64_t)c->nz + 2};
    const cuuint64_t strides[2] = {(cuuint64_t)c->pitch * 4, (cuuint64_t)c->plane * 4};
    const cuuint32_t box[3] = {box_x, box_y, 1};
    const cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(base), dims,
                     strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

// Grids the two-step kernel's boxes fit (136 x (TY + 4) rows at most).
bool tb_shape_ok(const ws3d_ctx* c) { return c->pitch >= 160 && c->H >= (uint32_t)kTbTY + 4; }

bool encode_buffer_maps(ws3d_ctx* c, int b) {
    return encode_slab_map(c, &c->mapP[b], c->buf[b], TmaLayout<kTmaTY, true>::kPRow,
                           kTmaTY + 2) &&
           encode_slab_map(c, &c->mapT[b], c->buf[b], 128, kTmaTY) &&
           // two-step pressure role: every ghost plane (tensor z = plane + gd)
           (!tb_shape_ok(c) ||
            (encode_slab_map(c, &c->mapA[b], fbuf_base(c, b), kTbRow, kTbTY + 4,
                             (uint64_t)c->nz + 2 * c->gd) &&
             encode_slab_map(c, &c->mapB[b], c->buf[b], kTbRow, kTbTY + 2)));
}

void build_tma_maps(ws3d_ctx* c) {
    c->tma_maps = false;
    if (c->pitch < 160 || c->H < 16) return;   // the kernel's boxes need W > 128, H >= 16
    bool ok = true;
    for (int b = 0; b < 2; ++b) ok = ok && encode_buffer_maps(c, b);
    c->tma_maps = ok;
}

void build_tma_c2_map(ws3d_ctx* c) {
    c->tma_c2_map = c->c2f && c->tma_maps &&
                    encode_slab_map(c, &c->mapC2, c->c2f, 128, kTmaTY) &&
                    (!tb_shape_ok(c) || encode_slab_map(c, &c->mapC2b, c->c2f, kTbRow, kTbTY + 2));
}

// The TMA kernel serves one GPU and z-slabs (its loads read only this GPU's
// memory; the ghost planes are local buffers written by the neighbours).
bool tma_eligible(const ws3d_ctx* c) {
    return c->cells_default && c->tma_maps && (!c->c2f || c->tma_c2_map);
}

template <bool kC2F, bool kLean>
ws3d_status launch_tma_t(ws3d_ctx* c, const StepParams& a) {
    using L = TmaLayout<kTmaTY, kC2F>;
    constexpr int kThreads = 32 * (kTmaTY + 1);
    const int smem = L::smem_bytes(kTmaStages);
    auto kern = k_step_tma<kC2F, kTmaTY, kLean>;
    int& grid = c->tma_grid[(kC2F ? 1 : 0) + (kLean ? 2 : 0)];
    if (grid == 0) {
        cudaError_t e =
            cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return cuda_fail(c, WS3D_ELAUNCH, e, "cudaFuncSetAttribute(tma)");
        int per_sm = 0;
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kThreads, smem);
        if (e != cudaSuccess || per_sm < 1)
            return cuda_fail(c, WS3D_ELAUNCH, e, "occupancy(tma)");
        grid = per_sm * std::max(1, c->sm_count);
    }
    const uint32_t tiles_x = (c->pitch + 127) / 128;
    const uint32_t tiles = tiles_x * ((c->H + kTmaTY - 1) / kTmaTY);
    // slabs: shorter chunks, so that interior chunks overlap the exchange
    const TmaSchedule sch =
        tma_schedule(tiles, c->nz, (uint32_t)grid, c->halo ? std::min(16u, c->tma_min_chunk)
                                                           : c->tma_min_chunk);
    const int P = c->ip, T = c->ipp;
    kern<<<sch.grid, kThreads, smem, c->stream>>>(c->mapP[P], c->mapT[T], c->mapC2, a, tiles_x,
                                                  tiles, sch.clen, sch.nitems);
    return check_launch(c, "k_step_tma");
}

template <bool kC2F>
ws3d_status launch_tma(ws3d_ctx* c, const StepParams& a) {
    return c->sponge_monotone ? launch_tma_t<kC2F, true>(c, a) : launch_tma_t<kC2F, false>(c, a);
}

// ---- two steps per launch (one GPU, default face layout) --------------------
// Buffers 2 and 3 hold no state between calls: a two-step launch writes
// p_{t+1} and p_{t+2} into them, then buf[] and the maps are permuted so that
// buffers 0 and 1 are again (pressure, pressure_prev).  Their ghost planes
// stay zero (one GPU: nothing writes them).
bool ensure_tb_buffers(ws3d_ctx* c) {
    if (c->tb_buffers) return true;
    if (c->tb_failed) return false;
    for (int b = 2; b < 4; ++b) {
        if (!c->buf[b] && falloc(c, b, "pressure (two-step)") != WS3D_OK) {
            cudaGetLastError();
            c->err.clear();
            c->tb_failed = true;
            return false;
        }
        if (!encode_buffer_maps(c, b)) {
            c->tb_failed = true;
            return false;
        }
    }
    c->tb_buffers = true;
    return true;
}

// The kernel's preconditions apart from the source count.
bool tb_kernel_ok(ws3d_ctx* c) {
    return tma_eligible(c) && tb_shape_ok(c) && c->sponge_monotone &&
           c->sponge_w <= (uint32_t)kTbSpongeMax &&
           (!c->c2f || c->tma_c2_map) && ensure_tb_buffers(c);
}

bool two_step_variant(const ws3d_ctx* c) {
    return c->desc.variant == WS3D_VARIANT_TMA2 || c->desc.variant == WS3D_VARIANT_AUTO;
}

// WS3D_HALO_CAP_* of this context (allocates the two-step buffers).
uint32_t halo_caps(ws3d_ctx* c) {
    uint32_t caps = 0;
    if (two_step_variant(c) && c->nz >= 2 && tb_kernel_ok(c)) caps |= WS3D_HALO_CAP_TWO_STEP;
    if (c->c2f) caps |= WS3D_HALO_CAP_C2_FIELD;
    return caps;
}

// TMA stages of the two-step kernel: five while a field (this context's
// planes) takes at most 1.5 GiB, four above.  Measured on B200 (C3 recipe,
// µs per launch, 4 / 5 stages): 512^3 517.6 / 495.1, 640^3 1005.6 / 959.5,
// 768x768x512 1131.9 / 1086.8, 896x896x256 772.0 / 727.9, 960x960x256
// 939.7 / 910.7, 1024x1024x256 1019.3 / 1011.6 -- but 768x768x1024 (2.4 GB a
// field) 2310.4 / 2399.7 and 1024^3 (4.3 GB) 4131.7 / 4513.3: the loss
// follows the size of the grid, not the width of its rows.
// WS3D_TWO_STEP_STAGES (4 or 5) at create overrides.
int tb_stages(const ws3d_ctx* c) {
    if (c->tb_stages_env) return c->tb_stages_env;
    return (uint64_t)c->pitch * c->H * c->nz * 4u <= (3ull << 29) ? kTbStagesHi : kTbStagesLo;
}

template <bool kC2F, int kS>
ws3d_status launch_tb_stages(ws3d_ctx* c) {
    using L = TbLayout<kC2F, kS>;
    constexpr int kThreads = 32 * (kTbTY + 3);
    const int smem = L::smem_bytes();
    // one GPU and z-slabs run separate instances (the slab code stays out
    // of the one-GPU item loop)
    auto kern = c->halo ? k_step_tma2<kC2F, true, kS> : k_step_tma2<kC2F, false, kS>;
    int& grid = c->tb_grid[(kC2F ? 1 : 0) + (c->halo ? 2 : 0) + (kS == kTbStagesHi ? 4 : 0)];
    if (grid == 0) {
        cudaError_t e =
            cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return cuda_fail(c, WS3D_ELAUNCH, e, "cudaFuncSetAttribute(tma2)");
        int per_sm = 0;
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kThreads, smem);
        if (e != cudaSuccess || per_sm < 1)
            return cuda_fail(c, WS3D_ELAUNCH, e, "occupancy(tma2)");
        grid = per_sm * std::max(1, c->sm_count);
    }
    TbArgs g{};
    g.a = make_params(c);
    g.X = owned0(c, c->buf[2]);
    g.Y = owned0(c, c->buf[3]);
    g.src_off = c->halo ? c->tb_src_off : c->src_off;
    g.wavelet = c->halo ? c->tb_wavelet : c->wavelet;
    g.n_src = c->halo ? c->tb_n_src : c->n_src;
    g.wl_len = c->wl_len;
    g.step1 = c->step + 1;
    g.a_zoff = (int)c->gd;
    // neighbours' own p_{t-1} (role ipp) and c2 planes next to ours come by
    // TMA through the peer maps; Y goes into their Y buffers (index 3, same
    // role on every rank).  One GPU: the own maps stand in (never read).
    const CUtensorMap* mbl = &c->mapB[c->ipp];
    const CUtensorMap* mbh = &c->mapB[c->ipp];
    const CUtensorMap* mcl = &c->mapC2b;
    const CUtensorMap* mch = &c->mapC2b;
    if (c->halo) {
        if (!c->peer_maps)
            return fail(c, WS3D_EPEER, "two-step slab launch without tensor maps of the neighbours");
        if (c->lo_base[0]) {
            g.has_lo = 1;
            g.lo_nz = c->lo_nz;
            g.peer_lo_y = c->lo_base[3] + c->lo_ghost_off;
            mbl = &c->mapBlo[c->ipp];
            if (kC2F) mcl = &c->mapC2lo;
        }
        if (c->hi_base[0]) {
            g.has_hi = 1;
            g.peer_hi_y = c->hi_base[3];
            mbh = &c->mapBhi[c->ipp];
            if (kC2F) mch = &c->mapC2hi;
        }
    }
    g.tiles_x = (c->pitch + 127) / 128;
    g.tiles = g.tiles_x * ((c->H + kTbTY - 1) / kTbTY);
    const TmaSchedule sch = tb_schedule(g.tiles, c->nz, (uint32_t)grid);
    g.clen = sch.clen;
    g.nitems = sch.nitems;
    kern<<<sch.grid, kThreads, smem, c->stream>>>(c->mapA[c->ip], c->mapB[c->ipp], c->mapC2b, *mbl,
                                                  *mbh, *mcl, *mch, g);
    ws3d_status s = check_launch(c, "k_step_tma2");
    if (s != WS3D_OK) return s;
    c->tb_launches++;
    // New roles: buffer 3 (p_{t+2}) is the pressure, buffer 2 (p_{t+1}) the
    // previous pressure; the old pair becomes the free pair.
    const int order[4] = {3, 2, c->ip, c->ipp};
    float *nb[4], *nlo[4], *nhi[4];
    CUtensorMap nP[4], nT[4], nA[4], nB[4], nBl[4], nBh[4];
    for (int k = 0; k < 4; ++k) {
        nb[k] = c->buf[order[k]];
        nlo[k] = c->lo_base[order[k]];
        nhi[k] = c->hi_base[order[k]];
        nP[k] = c->mapP[order[k]];
        nT[k] = c->mapT[order[k]];
        nA[k] = c->mapA[order[k]];
        nB[k] = c->mapB[order[k]];
        nBl[k] = c->mapBlo[order[k]];
        nBh[k] = c->mapBhi[order[k]];
    }
    for (int k = 0; k < 4; ++k) {
        c->buf[k] = nb[k];
        c->lo_base[k] = nlo[k];  // the neighbours permute theirs the same way
        c->hi_base[k] = nhi[k];
        c->mapP[k] = nP[k];
        c->mapT[k] = nT[k];
        c->mapA[k] = nA[k];
        c->mapB[k] = nB[k];
        c->mapBlo[k] = nBl[k];
        c->mapBhi[k] = nBh[k];
    }
    c->ip = 0;
    c->ipp = 1;
    return WS3D_OK;
}

template <bool kC2F>
ws3d_status launch_tb(ws3d_ctx* c) {
    return tb_stages(c) == kTbStagesHi ? launch_tb_stages<kC2F, kTbStagesHi>(c)
                                       : launch_tb_stages<kC2F, kTbStagesLo>(c);
}

// ---- cp.async kernel (one GPU or z-slabs, default face layout) -------------
template <bool kC2F>
ws3d_status launch_async(ws3d_ctx* c, const StepParams& a) {
    using L = AsyncLayout<kC2F>;
    constexpr int kThreads = 32 * (kAsyncTY + 1);
    const int smem = L::smem_bytes();
    int& resident = c->async_grid[kC2F ? 1 : 0];
    if (resident == 0) {
        cudaError_t e = cudaFuncSetAttribute(k_step_async<kC2F>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return cuda_fail(c, WS3D_ELAUNCH, e, "cudaFuncSetAttribute(async)");
        int per_sm = 0;
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_step_async<kC2F>, kThreads,
                                                          smem);
        if (e != cudaSuccess || per_sm < 1)
            return cuda_fail(c, WS3D_ELAUNCH, e, "occupancy(async)");
        resident = per_sm * std::max(1, c->sm_count);
    }
    AsyncSched sc{};
    sc.tiles_x = (c->pitch + 127) / 128;
    sc.tiles = sc.tiles_x * ((c->H + kAsyncTY - 1) / kAsyncTY);
    sc.nz = c->nz;
    sc.halo = a.wait_lo != nullptr || a.wait_hi != nullptr;
    const uint64_t field_bytes = (uint64_t)c->plane * c->nz * 4u * 3u;
    const uint32_t min_chunk = field_bytes <= (64ull << 20) ? 8u : c->tma_min_chunk;
    const TmaSchedule sch = tma_schedule(sc.tiles, c->nz, (uint32_t)resident, min_chunk);
    sc.clen = sch.clen;
    sc.nchunks = (c->nz + sch.clen - 1) / sch.clen;
    sc.nitems = sch.nitems;
    k_step_async<kC2F><<<sch.grid, kThreads, smem, c->stream>>>(a, sc);
    return check_launch(c, "k_step_async");
}

template <bool kC2F, bool kCells>
void launch_naive(const ws3d_ctx* c, const StepParams& a) {
    dim3 block(32, 4, 2);
    dim3 grid((c->W + 31) / 32, (c->H + 3) / 4, (c->nz + 1) / 2);
    k_step_naive<kC2F, kCells><<<grid, block, 0, c->stream>>>(a);
}

ws3d_status ensure_cell_arrays(ws3d_ctx* c);

// ---- persistent mode --------------------------------------------------------
constexpr int kPersTY = 8;

// Small one-GPU grids with the default faces and rows of at most 128 cells:
// the field stays in shared memory for the whole launch (k_persistent_smem,
// block shape from smem_step_shape, found once per context and c2 instance).
// False when the grid does not qualify.
template <bool kC2F>
bool smem_plan(ws3d_ctx* c) {
    if (!c->smem_persistent || c->halo || !c->cells_default || c->pitch > 128) return false;
    auto kern = k_persistent_smem<kC2F>;
    int& plan = c->smem_plan[kC2F ? 1 : 0];
    uint32_t& by = c->smem_by[kC2F ? 1 : 0];
    uint32_t& bz = c->smem_bz[kC2F ? 1 : 0];
    if (plan != 0) return plan > 0;
    plan = -1;
    if (!smem_step_shape(c->pitch, c->H, c->nz, (uint32_t)std::max(1, c->sm_count), kC2F,
                         (uint64_t)kSmemMaxBytes, &by, &bz))
        return false;
    const int want = (int)smem_step_bytes(c->pitch, by, bz, kC2F);
    // the attribute belongs to the function, not to this context: every
    // context sets the same bound (the kernel's maximum), so none lowers it
    // below another context's block size
    cudaError_t e =
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemMaxBytes);
    int per_sm = 0;
    if (e == cudaSuccess)
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kSmemThreads, want);
    const uint32_t blocks = ((c->H + by - 1) / by) * ((c->nz + bz - 1) / bz);
    if (e != cudaSuccess || per_sm < 1 || blocks > (uint32_t)(per_sm * std::max(1, c->sm_count))) {
        cudaGetLastError();
        return false;  // not co-resident here: the row body takes the launch
    }
    plan = 1;
    return true;
}

// Words of the exchange rows of a planned instance: two parities of
// 2 (by + bz) rows of pitch words per block.
size_t smem_xch_words(const ws3d_ctx* c, bool c2f) {
    const int k = c2f ? 1 : 0;
    const uint32_t by = c->smem_by[k], bz = c->smem_bz[k];
    const size_t blocks = (size_t)((c->H + by - 1) / by) * ((c->nz + bz - 1) / bz);
    return 2 * blocks * smem_xch_rows(by, bz) * c->pitch;
}

// Allocate (zeroed: tag 0 never matches) exchange rows of at least `words`;
// tags restart from the zeroed buffer.
ws3d_status smem_xch_alloc(ws3d_ctx* c, size_t words) {
    if (c->smem_xch_words < words) {
        dfree(c, c->smem_xch, c->smem_xch_words);
        c->smem_xch_words = 0;
        ws3d_status s = dalloc(c, &c->smem_xch, words, "shared-memory step exchange rows");
        if (s != WS3D_OK) return s;
        c->smem_xch_words = words;
    }
    WS3D_CUDA(c, cudaMemsetAsync(c->smem_xch, 0, c->smem_xch_words * sizeof *c->smem_xch, c->stream),
              WS3D_EMEMORY);
    c->smem_tag = 0;
    return WS3D_OK;
}

// At create: the exchange rows of both instances (with and without a c2
// field), so that stepping allocates nothing; a failure here only leaves the
// allocation to the first launch.
void smem_xch_prepare(ws3d_ctx* c) {
    if (c->nz != c->Dg) return;  // a z-slab: attached slabs take the row body
    size_t need = 0;
    if (smem_plan<false>(c)) need = std::max(need, smem_xch_words(c, false));
    if (smem_plan<true>(c)) need = std::max(need, smem_xch_words(c, true));
    if (need && smem_xch_alloc(c, need) != WS3D_OK) {
        cudaGetLastError();
        c->err.clear();
    }
}

template <bool kC2F>
ws3d_status launch_persistent_smem(ws3d_ctx* c, uint64_t n, bool* launched) {
    *launched = false;
    if (!smem_plan<kC2F>(c)) return WS3D_OK;
    const uint32_t by = c->smem_by[kC2F ? 1 : 0], bz = c->smem_bz[kC2F ? 1 : 0];
    const int bytes = (int)smem_step_bytes(c->pitch, by, bz, kC2F);
    const uint32_t yblocks = (c->H + by - 1) / by, zblocks = (c->nz + bz - 1) / bz;
    const uint32_t nblk = yblocks * zblocks;
    // exchange rows: allocated at create (smem_xch_prepare), here only when
    // that failed or a larger instance needs more; tags restart from a zeroed
    // buffer before the 32-bit tag would wrap
    if (n + 1 >= 0xffffffffull)
        return fail(c, WS3D_EINVAL, "step_persistent: at most 2^32 - 2 steps per launch");
    const size_t words = smem_xch_words(c, kC2F);
    if (c->smem_xch_words < words || (uint64_t)c->smem_tag + n + 1 >= 0xffffffffull) {
        ws3d_status s = smem_xch_alloc(c, words);
        if (s != WS3D_OK) return s;
    }
    SmemArgs q{};
    q.a = make_params(c);
    q.buf[0] = c->buf[c->ip];
    q.buf[1] = c->buf[c->ipp];
    q.xch = c->smem_xch;
    q.tag0 = c->smem_tag;
    c->smem_tag += (uint32_t)n;
    q.src_off = c->src_off;
    q.wavelet = c->wavelet;
    q.n_src = c->n_src;
    q.wl_len = c->wl_len;
    q.step0 = c->step;
    q.nsteps = n;
    q.by = by;
    q.bz = bz;
    q.yblocks = yblocks;
    q.zblocks = zblocks;
    void* args[] = {&q};
    cudaError_t e = cudaLaunchCooperativeKernel((const void*)k_persistent_smem<kC2F>, dim3(nblk),
                                                dim3(kSmemThreads),
                                                args, (size_t)bytes, c->stream);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return cuda_fail(c, WS3D_ELAUNCH, e, "cudaLaunchCooperativeKernel(k_persistent_smem)");
    }
    c->launches++;
    c->persistent_launches++;
    *launched = true;
    return WS3D_OK;
}

// Default face layout: the field in shared memory for small one-GPU grids
// (above), else the block-parallel body (k_persistent_rows, one L2 round trip
// per step); per-cell boundary arrays: the z-streaming body.
template <bool kC2F, bool kCells>
ws3d_status launch_persistent(ws3d_ctx* c, uint64_t n) {
    if constexpr (!kCells) {
        bool launched = false;
        ws3d_status s = launch_persistent_smem<kC2F>(c, n, &launched);
        if (s != WS3D_OK || launched) return s;
    }
    const void* kern = kCells ? (const void*)k_persistent<kC2F, kCells, kPersTY>
                              : (const void*)k_persistent_rows<kC2F>;
    const int threads = kCells ? 32 * kPersTY : kRowThreads;
    int& resident = c->pers_resident[(kC2F ? 2 : 0) + (kCells ? 1 : 0)];
    if (resident == 0) {
        int per_sm = 0;
        cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, threads, 0);
        if (e != cudaSuccess || per_sm < 1)
            return cuda_fail(c, WS3D_ELAUNCH, e, "occupancy(persistent)");
        resident = per_sm * std::max(1, c->sm_count);
    }
    PersistentArgs q{};
    q.a = make_params(c);
    q.a.peer_lo2 = q.a.peer_hi2 = nullptr;  // this kernel stores one plane per side
    // index 0 = pressure, 1 = pressure_prev at the start of the launch
    const int role[2] = {c->ip, c->ipp};
    for (int b = 0; b < 2; ++b) {
        q.buf[b] = c->buf[role[b]];
        q.lo_base[b] = c->lo_base[role[b] & 1];
        q.hi_base[b] = c->hi_base[role[b] & 1];
    }
    q.lo_ghost_off = c->lo_ghost_off;
    q.lo_flag = c->halo ? c->lo_flag : nullptr;
    q.hi_flag = c->halo ? c->hi_flag : nullptr;
    q.halo_base = c->halo_steps;
    q.bar = c->flags + kBarWord;
    // the barrier's arrival counter starts every launch at zero (stream order)
    WS3D_CUDA(c, cudaMemsetAsync(q.bar, 0, sizeof *q.bar, c->stream), WS3D_ELAUNCH);
    q.src_off = c->src_off;
    q.wavelet = c->wavelet;
    q.src_ghost = c->src_ghost;
    q.n_src = c->n_src;
    q.wl_len = c->wl_len;
    q.step0 = c->step;
    q.nsteps = n;
    q.cur0 = 0;
    q.tiles_x = (c->pitch + kZsTileX - 1) / kZsTileX;
    q.tiles = q.tiles_x * ((c->H + kPersTY - 1) / kPersTY);
    // Persistent launches are latency-bound per plane (small, L2-resident
    // grids): chunks down to 4 planes give every resident CTA work each step.
    const TmaSchedule sch = tma_schedule(q.tiles, c->nz, (uint32_t)resident, 4);
    q.clen = sch.clen;
    q.nitems = sch.nitems;
    void* args[] = {&q};
    // the row body: every co-resident CTA (rows are spread over all warps)
    const uint64_t rows = (uint64_t)c->nz * c->H * q.tiles_x;
    const uint64_t row_ctas = (rows + kRowThreads / 32 - 1) / (kRowThreads / 32);
    const dim3 grid = kCells ? dim3(sch.grid) : dim3((unsigned)std::min<uint64_t>(resident, row_ctas));
    const dim3 block = kCells ? dim3(32, kPersTY, 1) : dim3(kRowThreads, 1, 1);
    cudaError_t e = cudaLaunchCooperativeKernel(kern, grid, block, args, 0, c->stream);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return cuda_fail(c, e == cudaErrorCooperativeLaunchTooLarge ? WS3D_ELAUNCH : WS3D_ELAUNCH,
                         e, "cudaLaunchCooperativeKernel(k_persistent)");
    }
    c->launches++;
    c->persistent_launches++;
    return WS3D_OK;
}


ws3d_status launch_step(ws3d_ctx* c) {
    StepParams a = make_params(c);
    const bool f = a.c2f != nullptr;
    const bool cells = a.types != nullptr;
    uint32_t v = c->desc.variant;
    // auto (single steps; pairs of steps go to k_step_tma2, see use_two_step):
    // the TMA pipeline on one GPU and on z-slabs (0.91 of measured HBM peak at
    // 512^3 on one GPU); cell arrays and grids too narrow for its boxes take
    // the register-prefetch z-stream kernel (0.75), except small one-GPU
    // grids (each field at most 8 MiB, L2-resident), where one thread per cell
    // is faster than a few tiles walking z: at 64^3 3.8 us of kernel time per
    // step against 7.3 us (128^3: 12.8 against 13.7 us per launch).
    if (v == WS3D_VARIANT_AUTO) {
        const bool small = !c->halo && (uint64_t)c->pitch * c->H * c->nz * 4u <= (8ull << 20);
        v = tma_eligible(c) ? WS3D_VARIANT_TMA : small ? WS3D_VARIANT_NAIVE : WS3D_VARIANT_ZSTREAM;
    }
    if (v == WS3D_VARIANT_TMA2) v = WS3D_VARIANT_TMA;  // single steps of the two-step variant
    if (v == WS3D_VARIANT_ASYNC) {
        if (!c->cells_default)
            return fail(c, WS3D_EINVAL,
                        "the async kernel evaluates the default face layout only; use the auto "
                        "or zstream variant for per-cell boundary arrays");
        return f ? launch_async<true>(c, a) : launch_async<false>(c, a);
    }
    if (v == WS3D_VARIANT_TMA) {
        if (!tma_eligible(c))
            return fail(c, WS3D_EINVAL,
                        "the TMA kernel needs the default face layout, W > 128 and H >= 16; "
                        "use the auto or zstream variant");
        return f ? launch_tma<true>(c, a) : launch_tma<false>(c, a);
    }
    switch (v) {
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

// Per source: the offset of its cell in the lower neighbour's copy (relative
// to that buffer's plane -1) and in the upper one's (relative to its plane
// -2), or -1.  The neighbours hold copies of our first / last plane, and of
// the second / second-to-last one at temporal depth 2.
ws3d_status rebuild_source_ghosts(ws3d_ctx* c) {
    dfree(c, c->src_ghost, 2 * (size_t)c->n_src);
    if (!c->halo || c->n_src == 0) return WS3D_OK;
    std::vector<long long> gr(2 * (size_t)c->n_src, -1);
    bool any = false;
    const uint32_t depth = std::min(c->hdepth, c->nz);
    const long long P = (long long)c->plane;
    for (uint32_t k = 0; k < c->n_src; ++k) {
        const uint32_t x = c->src_xyz[3 * k], y = c->src_xyz[3 * k + 1], z = c->src_xyz[3 * k + 2];
        const long long row = (long long)y * c->pitch + x;
        const uint32_t from_lo = z - c->z0, from_hi = c->z0 + c->nz - 1 - z;  // 0 = edge plane
        if (c->lo_base[0] && from_lo < depth) {
            gr[2 * k] = (long long)c->lo_ghost_off + (long long)from_lo * P + row;
            any = true;
        }
        if (c->hi_base[0] && from_hi < depth) {
            gr[2 * k + 1] = (1 - (long long)from_hi) * P + row;  // plane -1 or -2
            any = true;
        }
    }
    if (!any) return WS3D_OK;
    ws3d_status s = dalloc(c, &c->src_ghost, gr.size(), "source ghosts");
    if (s != WS3D_OK) return s;
    WS3D_CUDA(c, cudaMemcpy(c->src_ghost, gr.data(), gr.size() * sizeof(long long),
                            cudaMemcpyHostToDevice),
              WS3D_EMEMORY);
    return WS3D_OK;
}

// The two-step kernel's source table on a z-slab at temporal depth 2: every
// source on planes -1 .. nz (its own and the ghost planes it computes p_{t+1}
// on), in the given order.
ws3d_status rebuild_tb_sources(ws3d_ctx* c) {
    dfree(c, c->tb_src_off, c->tb_n_src);
    dfree(c, c->tb_wavelet, (size_t)c->tb_n_src * c->wl_len);
    c->tb_n_src = 0;
    if (!c->halo || c->hdepth != 2 || c->n_src_global == 0) return WS3D_OK;
    std::vector<uint64_t> off;
    std::vector<float> wl;
    for (uint32_t k = 0; k < c->n_src_global; ++k) {
        const uint32_t x = c->gsrc_xyz[3 * k], y = c->gsrc_xyz[3 * k + 1], z = c->gsrc_xyz[3 * k + 2];
        if (z + 1 < c->z0 || z > c->z0 + c->nz) continue;
        off.push_back((uint64_t)(z + 1 - c->z0) * c->plane + (uint64_t)y * c->pitch + x);
        wl.insert(wl.end(), c->gsrc_wl.begin() + (size_t)k * c->wl_len,
                  c->gsrc_wl.begin() + (size_t)(k + 1) * c->wl_len);
    }
    if (off.empty()) return WS3D_OK;
    ws3d_status s;
    if ((s = dalloc(c, &c->tb_src_off, off.size(), "two-step sources")) != WS3D_OK) return s;
    if ((s = dalloc(c, &c->tb_wavelet, wl.size(), "two-step wavelet")) != WS3D_OK) return s;
    WS3D_CUDA(c, cudaMemcpy(c->tb_src_off, off.data(), off.size() * 8, cudaMemcpyHostToDevice),
              WS3D_EMEMORY);
    WS3D_CUDA(c, cudaMemcpy(c->tb_wavelet, wl.data(), wl.size() * 4, cudaMemcpyHostToDevice),
              WS3D_EMEMORY);
    c->tb_n_src = (uint32_t)off.size();
    return WS3D_OK;
}

// Sources of the next step; with `signal` (a z-slab with device-side flags)
// also raise the neighbours' flags for the next launch in the same kernel:
// this slab finished its previous launch (its stores into them, its reads of
// its own ghosts and of their planes) and this step's sources are in their
// copies.
ws3d_status launch_sources(ws3d_ctx* c, bool signal = false) {
    unsigned long long* flo = signal ? c->lo_flag : nullptr;
    unsigned long long* fhi = signal ? c->hi_flag : nullptr;
    const unsigned long long v = c->halo_steps + 1;
    if (!c->n_src) {
        if (!flo && !fhi) return WS3D_OK;
        k_halo_signal<<<1, 32, 0, c->stream>>>(flo, fhi, v);
        return check_launch(c, "k_halo_signal");
    }
    // neighbours' current pressure buffers (lower: plane -1, upper: plane -2)
    float* glo = c->lo_base[c->ip];
    float* ghi = c->hi_base[c->ip] ? c->hi_base[c->ip] - c->plane : nullptr;
    k_inject_sources<<<1, 32, 0, c->stream>>>(c->buf[c->ip], c->buf[c->ipp], c->src_off,
                                              c->wavelet, c->n_src, c->wl_len, c->step,
                                              c->src_ghost, glo, ghi, flo, fhi, v);
    return check_launch(c, "k_inject_sources");
}

// Read (and clear) the device status word the bounded waits write:
// bit 0 / 1 = wait for the lower / upper neighbour's flag, bit 2 = a stage
// wait of the TMA pipeline.
ws3d_status check_device_status(ws3d_ctx* c) {
    unsigned int st = 0;
    WS3D_CUDA(c, cudaMemcpy(&st, c->flags + 2, sizeof st, cudaMemcpyDeviceToHost), WS3D_EDEVICE);
    if (!st) return WS3D_OK;
    WS3D_CUDA(c, cudaMemset(c->flags + 2, 0, sizeof(unsigned long long)), WS3D_EDEVICE);
    if (st & 3u)
        return fail(c, WS3D_ETIMEOUT,
                    "a step gave up waiting for the %s%s%s neighbour after %.3f s (its flag "
                    "never reached the step); the field of that step is not valid",
                    (st & 1u) ? "lower" : "", (st & 3u) == 3u ? " and " : "",
                    (st & 2u) ? "upper" : "", c->budget_ns * 1e-9);
    return fail(c, WS3D_ETIMEOUT,
                "a pipeline stage wait gave up (status 0x%x); the field of that step is "
                "not valid", st);
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
    if (d->variant > WS3D_VARIANT_TMA2) { *why = "unknown variant"; return false; }
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
    c->gd = c->nz < c->Dg ? 2u : 1u;  // z-slab: room for temporal depth 2

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
        if ((s = falloc(c, b, "pressure")) != WS3D_OK) return bail(s);
    if (desc->sponge_width > 0) {
        c->sponge_w = desc->sponge_width;
        std::vector<float> tab(c->sponge_w);
        for (uint32_t d = 0; d < c->sponge_w; ++d) {
            const double t = (double)(c->sponge_w - d) / (double)c->sponge_w;
            tab[d] = (float)(1.0 - (double)desc->sponge_max * t * t);
        }
        for (uint32_t d = 0; d < c->sponge_w; ++d)
            if (!(tab[d] <= 1.0f) || (d + 1 < c->sponge_w && !(tab[d] <= tab[d + 1])))
                c->sponge_monotone = false;
        if ((s = dalloc(c, &c->sponge, c->sponge_w, "sponge")) != WS3D_OK) return bail(s);
        e = cudaMemcpy(c->sponge, tab.data(), tab.size() * sizeof(float), cudaMemcpyHostToDevice);
        if (e != cudaSuccess) return bail(cuda_fail(c, WS3D_EMEMORY, e, "cudaMemcpy(sponge)"));
    }
    if ((s = dalloc(c, &c->flags, kFlagWords, "halo flags")) != WS3D_OK) return bail(s);
    e = cudaMemsetAsync(c->flags, 0, kFlagWords * sizeof(unsigned long long), c->stream);
    if (e != cudaSuccess) return bail(cuda_fail(c, WS3D_EMEMORY, e, "cudaMemsetAsync(flags)"));
    if (desc->spin_budget) c->budget_ns = desc->spin_budget;
    if (const char* mc = getenv("WS3D_TMA_MIN_CHUNK")) {
        const long v = strtol(mc, nullptr, 10);
        if (v >= 1 && v <= (1 << 20)) c->tma_min_chunk = (uint32_t)v;
    }
    if (const char* ps = getenv("WS3D_PERSISTENT_SMEM")) c->smem_persistent = atoi(ps) != 0;
    if (const char* ts = getenv("WS3D_TWO_STEP_STAGES")) {
        const int v = atoi(ts);
        if (v == kTbStagesLo || v == kTbStagesHi) c->tb_stages_env = v;
    }
    build_tma_maps(c);
    // likewise the persistent shared-memory kernel's exchange rows
    smem_xch_prepare(c);
    // The two-step buffers are part of the auto / tma2 working set: allocate
    // them with the fields, not inside the first step (a failure only leaves
    // the context on single steps).
    if (two_step_variant(c) && c->tma_maps && c->sponge_monotone &&
        c->sponge_w <= (uint32_t)kTbSpongeMax)
        ensure_tb_buffers(c);
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
        // a resident kernel is told to terminate first (bounded wait)
        if (c->res_active) ws3d_resident_shutdown(c, 10000000000ull);
        // Never dereference a caller's stream here (it may already be gone):
        // wait for our own stream, or for the device when an external one is set.
        if (c->stream == c->own_stream) {
            if (c->own_stream) cudaStreamSynchronize(c->own_stream);
        } else {
            cudaDeviceSynchronize();
        }
        for (int b = 0; b < 4; ++b) ffree(c, b);
        dfree(c, c->c2f, c->slab);
        dfree(c, c->types, c->slab);
        dfree(c, c->refl, c->slab);
        dfree(c, c->sponge, c->sponge_w);
        dfree(c, c->src_off, c->n_src);
        dfree(c, c->wavelet, (size_t)c->n_src * c->wl_len);
        dfree(c, c->red_scratch, (size_t)c->red_blocks + 1);
        dfree(c, c->src_ghost, 2 * (size_t)c->n_src);
        dfree(c, c->tb_src_off, c->tb_n_src);
        dfree(c, c->tb_wavelet, (size_t)c->tb_n_src * c->wl_len);
        dfree(c, c->flags, kFlagWords);
        dfree(c, c->smem_xch, c->smem_xch_words);
        for (void* q : c->ipc_opened) cudaIpcCloseMemHandle(q);
        for (cudaEvent_t ev : c->tev) cudaEventDestroy(ev);
        dfree(c, c->vol16, c->vol_elems);
        dfree(c, c->img, c->img_elems);
        if (c->res_mem) cudaFreeHost(c->res_mem);
        if (c->res_done) cudaEventDestroy(c->res_done);
        if (c->res_side) cudaStreamDestroy(c->res_side);
        c->ipc_opened.clear();
        if (c->own_stream) cudaStreamDestroy(c->own_stream);
    }
    delete c;
}

const char* ws3d_last_error(const ws3d_ctx* c) { return c ? c->err.c_str() : ""; }

ws3d_status ws3d_upload(ws3d_ctx* c, const float* p, const float* pp) {
    WS3D_NOT_RESIDENT(c);
    if (!c) return WS3D_EINVAL;
    NvtxRange nv("ws3d.upload", kNvtxTransfer);
    DeviceGuard g(c->desc.device);
    ws3d_status s = WS3D_OK;
    if (p && (s = h2d_pitched(c, c->buf[c->ip], p)) != WS3D_OK) return s;
    if (pp && (s = h2d_pitched(c, c->buf[c->ipp], pp)) != WS3D_OK) return s;
    if (p) c->halo_synced = false;
    WS3D_CUDA(c, cudaStreamSynchronize(c->stream), WS3D_EMEMORY);
    return WS3D_OK;
}

ws3d_status ws3d_download(ws3d_ctx* c, float* p, float* pp) {
    WS3D_NOT_RESIDENT(c);
    if (!c || !p) return c ? fail(c, WS3D_EINVAL, "download: pressure is NULL") : WS3D_EINVAL;
    NvtxRange nv("ws3d.download", kNvtxTransfer);
    DeviceGuard g(c->desc.device);
    ws3d_status s = d2h_pitched(c, p, c->buf[c->ip], WS3D_EMEMORY);
    if (s == WS3D_OK && pp) s = d2h_pitched(c, pp, c->buf[c->ipp], WS3D_EMEMORY);
    if (s != WS3D_OK) return s;
    WS3D_CUDA(c, cudaStreamSynchronize(c->stream), WS3D_EMEMORY);
    return WS3D_OK;
}

ws3d_status ws3d_reset(ws3d_ctx* c, const float* p, const float* pp) {
    WS3D_NOT_RESIDENT(c);
    if (!c) return WS3D_EINVAL;
    c->ip = 0;
    c->ipp = 1;
    c->step = 0;
    c->halo_synced = false;
    DeviceGuard g(c->desc.device);
    for (int b = 0; b < 2; ++b)
        WS3D_CUDA(c, cudaMemsetAsync(fbuf_base(c, b), 0, fbuf_elems(c) * sizeof(float), c->stream),
                  WS3D_EMEMORY);
    return ws3d_upload(c, p, pp);
}

ws3d_status ws3d_set_cells(ws3d_ctx* c, const uint8_t* types, const float* refl) {
    WS3D_NOT_RESIDENT(c);
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
    if (c->halo && c->hdepth == 2)
        return fail(c, WS3D_ECOMMAND,
                    "set_cells: temporal depth 2 runs the TMA kernels, which take the default "
                    "face layout only; set depth 1 first");
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
    WS3D_NOT_RESIDENT(c);
    if (!c) return WS3D_EINVAL;
    if (c->halo && c->hdepth == 2 && (c2 == nullptr) != (c->c2f == nullptr))
        return fail(c, WS3D_ECOMMAND,
                    "set_c2_field: at temporal depth 2 the neighbours read this slab's c2 "
                    "planes; set the field before ws3d_halo_export, and keep it");
    DeviceGuard g(c->desc.device);
    if (!c2) {
        WS3D_CUDA(c, cudaStreamSynchronize(c->stream), WS3D_EDEVICE);
        dfree(c, c->c2f, c->slab);
        c->tma_c2_map = false;
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
    build_tma_c2_map(c);
    return WS3D_OK;
}

ws3d_status ws3d_set_sources(ws3d_ctx* c, uint32_t n, const uint32_t* xyz, const float* wavelet,
                             uint64_t len) {
    WS3D_NOT_RESIDENT(c);
    if (!c) return WS3D_EINVAL;
    if (n > 0 && (!xyz || !wavelet || len == 0))
        return fail(c, WS3D_EINVAL, "set_sources: xyz/wavelet missing");
    if (n > 65536) return fail(c, WS3D_EINVAL, "set_sources: more than 65536 sources");
    for (uint32_t k = 0; k < n; ++k)
        if (xyz[3 * k] >= c->W || xyz[3 * k + 1] >= c->H || xyz[3 * k + 2] >= c->Dg)
            return fail(c, WS3D_EINVAL, "set_sources: source %u at (%u,%u,%u) outside the grid",
                        k, xyz[3 * k], xyz[3 * k + 1], xyz[3 * k + 2]);
    DeviceGuard g(c->desc.device);
    WS3D_CUDA(c, cudaStreamSynchronize(c->stream), WS3D_EDEVICE);
    dfree(c, c->src_off, c->n_src);
    dfree(c, c->wavelet, (size_t)c->n_src * c->wl_len);
    dfree(c, c->src_ghost, 2 * (size_t)c->n_src);
    dfree(c, c->tb_src_off, c->tb_n_src);
    dfree(c, c->tb_wavelet, (size_t)c->tb_n_src * c->wl_len);
    c->n_src = 0;
    c->tb_n_src = 0;
    c->wl_len = n ? len : 0;
    c->src_xyz.clear();
    // the whole list, for the ghost planes of two-step launches on z-slabs
    c->n_src_global = n;
    c->gsrc_xyz.assign(xyz, xyz + 3 * (size_t)n);
    c->gsrc_wl.assign(wavelet, wavelet + (size_t)n * (n ? len : 0));
    // Keep only the sources inside the owned planes, in their given order.
    std::vector<uint64_t> off;
    std::vector<float> wl;
    for (uint32_t k = 0; k < n; ++k) {
        const uint32_t x = xyz[3 * k], y = xyz[3 * k + 1], z = xyz[3 * k + 2];
        if (z < c->z0 || z >= c->z0 + c->nz) continue;
        off.push_back((uint64_t)(z - c->z0 + 1) * c->plane + (uint64_t)y * c->pitch + x);
        wl.insert(wl.end(), wavelet + (size_t)k * len, wavelet + (size_t)(k + 1) * len);
        c->src_xyz.insert(c->src_xyz.end(), {x, y, z});
    }
    ws3d_status s;
    if (!off.empty()) {
        if ((s = dalloc(c, &c->src_off, off.size(), "sources")) != WS3D_OK) return s;
        if ((s = dalloc(c, &c->wavelet, wl.size(), "wavelet")) != WS3D_OK) return s;
        WS3D_CUDA(c, cudaMemcpy(c->src_off, off.data(), off.size() * 8, cudaMemcpyHostToDevice),
                  WS3D_EMEMORY);
        WS3D_CUDA(c, cudaMemcpy(c->wavelet, wl.data(), wl.size() * 4, cudaMemcpyHostToDevice),
                  WS3D_EMEMORY);
        c->n_src = (uint32_t)off.size();
    }
    if ((s = rebuild_source_ghosts(c)) != WS3D_OK) return s;
    return rebuild_tb_sources(c);
}

namespace {
// Two steps per launch for the auto and tma2 variants where the context
// allows it (default faces, TMA maps, at most 32 sources, a monotone sponge
// of width <= 64, memory for two more field buffers); otherwise single
// steps.  Measured on B200 at 512^3 (c2 field, sponge): 0.64 ms per two-step
// launch against 2 x 0.359 ms for two TMA steps.  On z-slabs only at
// temporal depth 2, and by a rule every rank evaluates alike (the whole
// source list, not this slab's share, decides), so that all ranks take the
// same launches; the neighbours must hold our two edge planes (not so right
// after persistent steps, which store one).
bool use_two_step(ws3d_ctx* c) {
    if (!two_step_variant(c)) return false;
    if (c->halo)
        return c->hdepth == 2 && c->deep_ok && c->n_src_global <= (uint32_t)kTbMaxSrc &&
               tb_kernel_ok(c);
    return c->n_src <= (uint32_t)kTbMaxSrc && tb_kernel_ok(c);
}

// Timed launches keep their event pairs in a ring of kTimedRing slots: a
// slot is reused only after the pair recorded in it kTimedRing launches
// earlier has been read (the host waits for that old launch, which leaves
// kTimedRing - 1 launches queued), so the event count stays bounded.
constexpr uint64_t kTimedRing = 256;

// Sum the elapsed time of up to `max` of the oldest unread pairs into tev_ms.
ws3d_status timed_fold(ws3d_ctx* c, uint64_t max) {
    for (; c->tev_done < c->tev_rec && max > 0; --max) {
        const size_t slot = (size_t)(c->tev_done % kTimedRing);
        WS3D_CUDA(c, cudaEventSynchronize(c->tev[2 * slot + 1]), WS3D_ELAUNCH);
        float ms = 0.f;
        WS3D_CUDA(c, cudaEventElapsedTime(&ms, c->tev[2 * slot], c->tev[2 * slot + 1]),
                  WS3D_EDEVICE);
        c->tev_ms += ms;
        c->tev_done++;
    }
    return WS3D_OK;
}

// Record the start (end = false) or end event of timed launch tev_rec.
ws3d_status timed_mark(ws3d_ctx* c, bool end) {
    const size_t slot = (size_t)(c->tev_rec % kTimedRing);
    if (!end) {
        if (c->tev_rec - c->tev_done >= kTimedRing) {
            ws3d_status s = timed_fold(c, 1);
            if (s != WS3D_OK) return s;
        }
        while (c->tev.size() < 2 * (slot + 1)) {
            cudaEvent_t ev;
            WS3D_CUDA(c, cudaEventCreate(&ev), WS3D_EDEVICE);
            c->tev.push_back(ev);
        }
    }
    WS3D_CUDA(c, cudaEventRecord(c->tev[2 * slot + (end ? 1 : 0)], c->stream), WS3D_EDEVICE);
    if (end) c->tev_rec++;
    return WS3D_OK;
}

// Advances n steps; with `timed`, records an event pair around every step
// launch (timed_mark).
ws3d_status step_impl(ws3d_ctx* c, uint64_t n, bool timed) {
    if (c->halo && c->host_ordered)
        return fail(c, WS3D_ECOMMAND, "step: same-device slabs advance through ws3d_step_group");
    if (c->halo && !c->halo_synced)
        return fail(c, WS3D_ECOMMAND, "step: fields changed since the last ws3d_halo_sync");
    if (c->halo && c->hdepth == 2 && !tma_eligible(c))
        return fail(c, WS3D_ECOMMAND,
                    "step: temporal depth 2 needs the TMA kernels (default faces, W > 128, H >= 16)");
    // Several steps of a small one-GPU grid (variant auto, default faces, rows
    // of at most 128 cells, the field fits the SMs' shared memory): one launch
    // of k_persistent_smem instead of a latency-bound launch per step --
    // bit-identical (same rule, same order, sources applied per step), and at
    // 64^3 4.2 us per step against 8.8 us of kernel time per single-step launch.
    if (n >= 2 && !c->halo && c->desc.variant == WS3D_VARIANT_AUTO) {
        ws3d_status s;
        if (timed && (s = timed_mark(c, false)) != WS3D_OK) return s;
        bool launched = false;
        s = c->c2f ? launch_persistent_smem<true>(c, n, &launched)
                   : launch_persistent_smem<false>(c, n, &launched);
        if (s != WS3D_OK) return s;
        if (launched) {
            if (timed && (s = timed_mark(c, true)) != WS3D_OK) return s;
            if (n & 1u) std::swap(c->ip, c->ipp);
            c->step += n;
            c->halo_steps += n;
            return WS3D_OK;
        }
        // not eligible: the start event recorded above is recorded again below
    }
    for (uint64_t i = 0; i < n;) {
        // sources of this step and, on slabs, the one signal per launch that
        // lets the neighbours' next launch start
        ws3d_status s = launch_sources(c, c->halo);
        if (s != WS3D_OK) return s;
        const bool two = n - i >= 2 && use_two_step(c);
        if (timed && (s = timed_mark(c, false)) != WS3D_OK) return s;
        if (two) {
            // sources of step t went into A and B above; the kernel applies
            // those of step t+1 between its two steps
            s = c->c2f ? launch_tb<true>(c) : launch_tb<false>(c);
        } else if ((s = launch_step(c)) == WS3D_OK) {
            std::swap(c->ip, c->ipp);
        }
        if (s != WS3D_OK) return s;
        if (timed && (s = timed_mark(c, true)) != WS3D_OK) return s;
        c->step += two ? 2 : 1;
        i += two ? 2 : 1;
        c->halo_steps++;
        c->deep_ok = true;  // both launches store two edge planes at temporal depth 2
    }
    return WS3D_OK;
}
}  // namespace

ws3d_status ws3d_step(ws3d_ctx* c, uint64_t n) {
    WS3D_NOT_RESIDENT(c);
    if (!c) return WS3D_EINVAL;
    NvtxRange nv("ws3d.steps", kNvtxKernel);
    DeviceGuard g(c->desc.device);
    return step_impl(c, n, false);
}

ws3d_status ws3d_step_timed_begin(ws3d_ctx* c, uint64_t n) {
    WS3D_NOT_RESIDENT(c);
    if (!c) return WS3D_EINVAL;
    if (n > (1u << 20)) return fail(c, WS3D_EINVAL, "step_timed: more than 2^20 steps");
    NvtxRange nv("ws3d.steps_timed", kNvtxKernel);
    DeviceGuard g(c->desc.device);
    c->tev_rec = c->tev_done = 0;
    c->tev_ms = 0.0;
    return step_impl(c, n, true);
}

ws3d_status ws3d_step_timed_end(ws3d_ctx* c, double* kernel_ms) {
    WS3D_NOT_RESIDENT(c);
    if (!c || !kernel_ms) return c ? fail(c, WS3D_EINVAL, "step_timed: kernel_ms is NULL")
                                   : WS3D_EINVAL;
    DeviceGuard g(c->desc.device);
    WS3D_CUDA(c, cudaStreamSynchronize(c->stream), WS3D_ELAUNCH);
    ws3d_status s = timed_fold(c, c->tev_rec);
    if (s != WS3D_OK) return s;
    *kernel_ms = c->tev_ms;
    return check_device_status(c);
}

ws3d_status ws3d_step_timed(ws3d_ctx* c, uint64_t n, double* kernel_ms) {
    if (c && !kernel_ms) return fail(c, WS3D_EINVAL, "step_timed: kernel_ms is NULL");
    ws3d_status s = ws3d_step_timed_begin(c, n);
    return s != WS3D_OK ? s : ws3d_step_timed_end(c, kernel_ms);
}

ws3d_status ws3d_halo_wait_stats(ws3d_ctx* c, uint64_t* wait_ns, uint64_t* waits, int reset) {
    if (!c) return WS3D_EINVAL;
    DeviceGuard g(c->desc.device);
    unsigned long long v[2] = {0, 0};
    WS3D_CUDA(c, cudaStreamSynchronize(c->stream), WS3D_ELAUNCH);
    WS3D_CUDA(c, cudaMemcpy(v, c->flags + kWaitAccWord, sizeof v, cudaMemcpyDeviceToHost),
              WS3D_EDEVICE);
    if (wait_ns) *wait_ns = v[0];
    if (waits) *waits = v[1];
    if (reset)
        WS3D_CUDA(c, cudaMemset(c->flags + kWaitAccWord, 0, sizeof v), WS3D_EDEVICE);
    return WS3D_OK;
}

namespace {
// Add amp*factor to the listed cells (and amp*factor*0.5 to p_prev), and to
// the neighbours' ghost copies of the cells on the edge planes (pressure
// only: glo relative to the lower neighbour's first upper ghost plane, ghi
// relative to the upper one's plane -2).
ws3d_status apply_impulse_table(ws3d_ctx* c, const std::vector<uint64_t>& off,
                                const std::vector<float>& fac, const std::vector<uint64_t>& glo,
                                const std::vector<float>& flo, const std::vector<uint64_t>& ghi,
                                const std::vector<float>& fhi, float amp) {
    struct Part { const std::vector<uint64_t>* o; const std::vector<float>* f; float* ghost; };
    const Part parts[3] = {{&off, &fac, nullptr},
                           {&glo, &flo, c->lo_base[c->ip] ? c->lo_base[c->ip] + c->lo_ghost_off : nullptr},
                           {&ghi, &fhi, c->hi_base[c->ip] ? c->hi_base[c->ip] - c->plane : nullptr}};
    ws3d_status s = WS3D_OK;
    for (int k = 0; k < 3 && s == WS3D_OK; ++k) {
        const Part& q = parts[k];
        if (q.o->empty() || (k > 0 && !q.ghost)) continue;
        uint64_t* d_off = nullptr;
        float* d_fac = nullptr;
        if ((s = dalloc(c, &d_off, q.o->size(), "impulse offsets")) != WS3D_OK) return s;
        if ((s = dalloc(c, &d_fac, q.f->size(), "impulse factors")) != WS3D_OK) {
            dfree(c, d_off, q.o->size());
            return s;
        }
        cudaError_t e1 = cudaMemcpyAsync(d_off, q.o->data(), q.o->size() * 8,
                                         cudaMemcpyHostToDevice, c->stream);
        cudaError_t e2 = cudaMemcpyAsync(d_fac, q.f->data(), q.f->size() * 4,
                                         cudaMemcpyHostToDevice, c->stream);
        const uint32_t n = (uint32_t)q.o->size();
        if (e1 != cudaSuccess || e2 != cudaSuccess) {
            s = cuda_fail(c, WS3D_EMEMORY, e1 != cudaSuccess ? e1 : e2, "cudaMemcpyAsync(impulse)");
        } else if (k == 0) {
            k_inject_table<<<(n + 255) / 256, 256, 0, c->stream>>>(
                c->buf[c->ip], c->buf[c->ipp], d_off, d_fac, n, amp);
            s = check_launch(c, "k_inject_table");
        } else {
            k_inject_ghost<<<(n + 255) / 256, 256, 0, c->stream>>>(q.ghost, d_off, d_fac, n, amp);
            s = check_launch(c, "k_inject_ghost");
        }
        cudaStreamSynchronize(c->stream);
        dfree(c, d_off, q.o->size());
        dfree(c, d_fac, q.f->size());
    }
    return s;
}

// Collect (offset, factor) for the cells of an impulse that this slab owns.
struct ImpulseCells {
    std::vector<uint64_t> off, glo, ghi;
    std::vector<float> fac, flo, fhi;
    void add(const ws3d_ctx* c, uint32_t x, uint32_t y, uint32_t z, float f) {
        if (z < c->z0 || z >= c->z0 + c->nz) return;
        const uint64_t row = (uint64_t)y * c->pitch + x;
        off.push_back((uint64_t)(z - c->z0 + 1) * c->plane + row);
        fac.push_back(f);
        const uint32_t d = std::min(c->hdepth, c->nz);  // edge planes the neighbours hold
        const uint32_t from_lo = z - c->z0, from_hi = c->z0 + c->nz - 1 - z;
        if (from_lo < d && c->lo_base[0]) {
            glo.push_back(from_lo * c->plane + row);
            flo.push_back(f);
        }
        if (from_hi < d && c->hi_base[0]) {
            ghi.push_back((1 - from_hi) * c->plane + row);
            fhi.push_back(f);
        }
    }
};
}  // namespace

ws3d_status ws3d_inject_impulse(ws3d_ctx* c, uint32_t x, uint32_t y, uint32_t z, float amp) {
    WS3D_NOT_RESIDENT(c);
    if (!c) return WS3D_EINVAL;
    if (x >= c->W || y >= c->H || z >= c->Dg) return WS3D_OK;  // grid3d.rs:147
    if (z < c->z0 || z >= c->z0 + c->nz) return WS3D_OK;      // another slab owns it
    DeviceGuard g(c->desc.device);
    const uint64_t off = (uint64_t)(z - c->z0 + 1) * c->plane + (uint64_t)y * c->pitch + x;
    const uint32_t d = std::min(c->hdepth, c->nz);
    const bool on_lo = z - c->z0 < d && c->lo_base[0];
    const bool on_hi = c->z0 + c->nz - 1 - z < d && c->hi_base[0];
    if (!on_lo && !on_hi) {
        k_inject_point<<<1, 32, 0, c->stream>>>(c->buf[c->ip], c->buf[c->ipp], off, amp);
        return check_launch(c, "k_inject_point");
    }
    // amp * 1.0f == amp exactly, so the table path adds the same values.
    ImpulseCells cells;
    cells.add(c, x, y, z, 1.0f);
    return apply_impulse_table(c, cells.off, cells.fac, cells.glo, cells.flo, cells.ghi, cells.fhi,
                               amp);
}

ws3d_status ws3d_inject_spherical_impulse(ws3d_ctx* c, uint32_t cx, uint32_t cy, uint32_t cz,
                                          float amp, float radius) {
    WS3D_NOT_RESIDENT(c);
    if (!c) return WS3D_EINVAL;
    if (!(radius >= 0.0f) || radius > 1024.0f)
        return fail(c, WS3D_EINVAL, "inject_spherical_impulse: radius %g outside [0, 1024]",
                    (double)radius);
    DeviceGuard g(c->desc.device);
    const int r = (int)radius;
    const float r_sq = radius * radius;
    ImpulseCells cells;
    for (int dz = -r; dz <= r; ++dz)
        for (int dy = -r; dy <= r; ++dy)
            for (int dx = -r; dx <= r; ++dx) {
                const long long x = (long long)cx + dx, y = (long long)cy + dy,
                                z = (long long)cz + dz;
                if (x < 0 || y < 0 || z < 0 || x >= c->W || y >= c->H || z >= c->Dg) continue;
                const float dist_sq = (float)(dx * dx + dy * dy + dz * dz);
                if (!(dist_sq <= r_sq)) continue;
                cells.add(c, (uint32_t)x, (uint32_t)y, (uint32_t)z,
                          expf(-dist_sq / (2.0f * radius)));
            }
    if (cells.off.empty()) return WS3D_OK;
    return apply_impulse_table(c, cells.off, cells.fac, cells.glo, cells.flo, cells.ghi, cells.fhi,
                               amp);
}

ws3d_status ws3d_energy(ws3d_ctx* c, double* out) {
    WS3D_NOT_RESIDENT(c);
    if (!c || !out) return WS3D_EINVAL;
    DeviceGuard g(c->desc.device);
    const uint64_t rows = (uint64_t)c->nz * c->H;
    k_energy_partials<<<c->red_blocks, kRedThreads, 0, c->stream>>>(
        owned0(c, c->buf[c->ip]), c->W, c->pitch, rows, c->red_scratch);
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
    WS3D_NOT_RESIDENT(c);
    if (!c || !out) return WS3D_EINVAL;
    DeviceGuard g(c->desc.device);
    const uint64_t rows = (uint64_t)c->nz * c->H;
    float* part = reinterpret_cast<float*>(c->red_scratch);
    k_maxabs_partials<<<c->red_blocks, kRedThreads, 0, c->stream>>>(
        owned0(c, c->buf[c->ip]), c->W, c->pitch, rows, part);
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
    WS3D_NOT_RESIDENT(c);
    if (!c) return WS3D_EINVAL;
    DeviceGuard g(c->desc.device);
    WS3D_CUDA(c, cudaStreamSynchronize(c->stream), WS3D_ELAUNCH);
    return check_device_status(c);
}

ws3d_status ws3d_set_stream(ws3d_ctx* c, void* stream) {
    WS3D_NOT_RESIDENT(c);
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
    o->two_step_launches = (uint32_t)std::min<uint64_t>(c->tb_launches, 0xffffffffull);
    return WS3D_OK;
}


ws3d_status ws3d_step_persistent(ws3d_ctx* c, uint64_t n) {
    WS3D_NOT_RESIDENT(c);
    if (!c) return WS3D_EINVAL;
    NvtxRange nv("ws3d.steps_persistent", kNvtxKernel);
    if (c->halo && c->host_ordered)
        return fail(c, WS3D_ECOMMAND, "step_persistent: same-device slab groups step through "
                                      "ws3d_step_group");
    if (c->halo && !c->halo_synced)
        return fail(c, WS3D_ECOMMAND, "step_persistent: fields changed since the last halo sync");
    if (n == 0) return WS3D_OK;
    DeviceGuard g(c->desc.device);
    const bool f = c->c2f != nullptr, cells = !c->cells_default;
    ws3d_status s;
    if (f && cells) s = launch_persistent<true, true>(c, n);
    else if (f) s = launch_persistent<true, false>(c, n);
    else if (cells) s = launch_persistent<false, true>(c, n);
    else s = launch_persistent<false, false>(c, n);
    if (s != WS3D_OK) return s;
    if (n & 1u) std::swap(c->ip, c->ipp);
    c->step += n;
    c->halo_steps += n;
    c->deep_ok = false;  // one plane per side went to the neighbours: single steps next
    return WS3D_OK;
}

ws3d_status ws3d_get_slice(ws3d_ctx* c, uint32_t axis, uint32_t index, float* out) {
    WS3D_NOT_RESIDENT(c);
    if (!c || !out) return c ? fail(c, WS3D_EINVAL, "get_slice: out is NULL") : WS3D_EINVAL;
    DeviceGuard g(c->desc.device);
    const float* P = owned0(c, c->buf[c->ip]);
    cudaError_t e = cudaSuccess;
    if (axis == 0) {  // XY at z (grid3d.rs:414-418)
        const uint32_t z = std::min(index, c->Dg - 1);
        if (z < c->z0 || z >= c->z0 + c->nz)
            return fail(c, WS3D_EINVAL, "get_slice: plane z=%u is not owned by this slab", z);
        e = cudaMemcpy2DAsync(out, c->W * 4, P + (size_t)(z - c->z0) * c->plane, c->pitch * 4,
                              c->W * 4, c->H, cudaMemcpyDeviceToHost, c->stream);
    } else if (axis == 1) {  // XZ at y (grid3d.rs:421-430): one row per owned plane
        const uint32_t y = std::min(index, c->H - 1);
        e = cudaMemcpy2DAsync(out, c->W * 4, P + (size_t)y * c->pitch, c->plane * 4, c->W * 4,
                              c->nz, cudaMemcpyDeviceToHost, c->stream);
    } else if (axis == 2) {  // YZ at x (grid3d.rs:433-442): one float per (z, y)
        const uint32_t x = std::min(index, c->W - 1);
        e = cudaMemcpy2DAsync(out, 4, P + x, c->pitch * 4, 4, (size_t)c->H * c->nz,
                              cudaMemcpyDeviceToHost, c->stream);
    } else {
        return fail(c, WS3D_EINVAL, "get_slice: axis must be 0 (XY), 1 (XZ) or 2 (YZ)");
    }
    if (e != cudaSuccess) return cuda_fail(c, WS3D_EREADBACK, e, "get_slice copy");
    WS3D_CUDA(c, cudaStreamSynchronize(c->stream), WS3D_EREADBACK);
    return WS3D_OK;
}

ws3d_status ws3d_sample_pressure(ws3d_ctx* c, uint32_t n, const float* pos_m, float cell_size,
                                 float* out) {
    WS3D_NOT_RESIDENT(c);
    if (!c) return WS3D_EINVAL;
    if (n == 0) return WS3D_OK;
    if (!pos_m || !out || !(cell_size > 0.0f) || n > (1u << 24))
        return fail(c, WS3D_EINVAL, "sample_pressure: bad arguments");
    // Every sample's planes z0, z0+1 (clamped) must be readable by this context.
    for (uint32_t i = 0; i < n; ++i) {
        const float fz = pos_m[3 * i + 2] / cell_size;
        const float flz = floorf(fz);
        const uint32_t z0 = flz > 0.f ? (uint32_t)flz : 0u;
        const uint32_t zz0 = std::min(z0, c->Dg - 1), z1 = std::min(z0 + 1u, c->Dg - 1);
        const bool ok0 = zz0 >= c->z0 && zz0 < c->z0 + c->nz;
        const bool ok1 = (z1 >= c->z0 && z1 < c->z0 + c->nz) ||
                         (z1 == c->z0 + c->nz && c->halo && c->halo_synced && c->hi_base[0]);
        if (!ok0 || !ok1 || !(pos_m[3 * i] >= 0.f) || !(pos_m[3 * i + 1] >= 0.f) ||
            !(pos_m[3 * i + 2] >= 0.f) || pos_m[3 * i] / cell_size >= (float)c->W ||
            pos_m[3 * i + 1] / cell_size >= (float)c->H || fz >= (float)c->Dg)
            return fail(c, WS3D_EINVAL, "sample_pressure: sample %u is outside this context's cells", i);
    }
    DeviceGuard g(c->desc.device);
    float* d = nullptr;
    ws3d_status s = dalloc(c, &d, (size_t)n * 4, "samples");
    if (s != WS3D_OK) return s;
    cudaError_t e = cudaMemcpyAsync(d, pos_m, (size_t)n * 12, cudaMemcpyHostToDevice, c->stream);
    if (e == cudaSuccess) {
        k_sample<<<(n + 127) / 128, 128, 0, c->stream>>>(owned0(c, c->buf[c->ip]), c->W, c->H,
                                                         c->Dg, c->pitch, c->plane, c->z0, d,
                                                         cell_size, n, d + 3 * (size_t)n);
        s = check_launch(c, "k_sample");
        if (s == WS3D_OK)
            e = cudaMemcpyAsync(out, d + 3 * (size_t)n, (size_t)n * 4, cudaMemcpyDeviceToHost,
                                c->stream);
    }
    if (s == WS3D_OK && e != cudaSuccess) s = cuda_fail(c, WS3D_EREADBACK, e, "sample copy");
    cudaStreamSynchronize(c->stream);
    dfree(c, d, (size_t)n * 4);
    return s;
}

ws3d_status ws3d_set_step(ws3d_ctx* c, uint64_t step) {
    WS3D_NOT_RESIDENT(c);
    if (!c) return WS3D_EINVAL;
    DeviceGuard g(c->desc.device);
    WS3D_CUDA(c, cudaStreamSynchronize(c->stream), WS3D_EDEVICE);
    c->step = step;
    return WS3D_OK;
}

// ---------------------------------------------------------------------------
// z-slab halo exchange.
// ---------------------------------------------------------------------------
namespace {
// Called after the neighbours' pointers, caps and sizes are in place.
ws3d_status attach_common(ws3d_ctx* c) {
    c->halo = c->lo_base[0] != nullptr || c->hi_base[0] != nullptr;
    // tensor maps over the neighbours' buffers (two-step slabs; see mapBlo)
    c->peer_maps = c->halo && c->tma_maps && tb_shape_ok(c);
    for (int b = 0; b < 4 && c->peer_maps; ++b) {
        if (c->lo_base[b])
            c->peer_maps = encode_slab_map(c, &c->mapBlo[b], c->lo_base[b], kTbRow, kTbTY + 2,
                                           (uint64_t)c->lo_nz + 2);
        if (c->peer_maps && c->hi_base[b])
            c->peer_maps = encode_slab_map(c, &c->mapBhi[b], c->hi_base[b], kTbRow, kTbTY + 2,
                                           (uint64_t)c->hi_nz + 2);
    }
    if (c->peer_maps && c->lo_c2)
        c->peer_maps = encode_slab_map(c, &c->mapC2lo, c->lo_c2, kTbRow, kTbTY + 2,
                                       (uint64_t)c->lo_nz + 2);
    if (c->peer_maps && c->hi_c2)
        c->peer_maps = encode_slab_map(c, &c->mapC2hi, c->hi_c2, kTbRow, kTbTY + 2,
                                       (uint64_t)c->hi_nz + 2);
    c->halo_synced = false;
    c->halo_steps = 0;
    c->hdepth = 1;
    c->deep_ok = false;
    c->lo_ghost_off = c->lo_base[0] ? (uint64_t)(c->lo_nz + 1) * c->plane : 0;
    if (c->halo && c->desc.variant != WS3D_VARIANT_ZSTREAM &&
        c->desc.variant != WS3D_VARIANT_AUTO && c->desc.variant != WS3D_VARIANT_ASYNC &&
        c->desc.variant != WS3D_VARIANT_TMA && c->desc.variant != WS3D_VARIANT_TMA2)
        return fail(c, WS3D_EINVAL,
                    "halo exchange needs the auto, tma, tma2, async or zstream variant");
    ws3d_status s = rebuild_source_ghosts(c);
    return s == WS3D_OK ? rebuild_tb_sources(c) : s;
}

bool same_geometry(const ws3d_ctx* c, uint32_t W, uint32_t H, uint32_t D, uint32_t pitch) {
    return W == c->W && H == c->H && D == c->Dg && pitch == c->pitch;
}
}  // namespace

ws3d_status ws3d_halo_export(ws3d_ctx* c, ws3d_halo_handles* out) {
    WS3D_NOT_RESIDENT(c);
    if (!c || !out) return c ? fail(c, WS3D_EINVAL, "halo_export: out is NULL") : WS3D_EINVAL;
    NvtxRange nv("ws3d.connect.export", kNvtxSync);
    static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
    static_assert(sizeof(ws3d_halo_handles) == 424, "ws3d_halo_handles layout");
    DeviceGuard g(c->desc.device);
    std::memset(out, 0, sizeof *out);
    const uint32_t caps = halo_caps(c);  // two-step capable: buffers 2 and 3 exist now
    cudaIpcMemHandle_t h;
    const int nb = (caps & WS3D_HALO_CAP_TWO_STEP) ? 4 : 2;
    for (int b = 0; b < nb; ++b) {
        WS3D_CUDA(c, cudaIpcGetMemHandle(&h, fbuf_base(c, b)), WS3D_EPEER);
        std::memcpy(out->buf[b], &h, 64);
    }
    WS3D_CUDA(c, cudaIpcGetMemHandle(&h, c->flags), WS3D_EPEER);
    std::memcpy(out->flags, &h, 64);
    if (c->c2f) {
        WS3D_CUDA(c, cudaIpcGetMemHandle(&h, c->c2f), WS3D_EPEER);
        std::memcpy(out->c2, &h, 64);
    }
    out->width = c->W;
    out->height = c->H;
    out->depth = c->Dg;
    out->pitch = c->pitch;
    out->z_begin = c->z0;
    out->z_end = c->z0 + c->nz;
    out->device = c->desc.device;
    out->caps = caps;
    out->ghost_planes = c->gd;
    out->c_squared = c->desc.c_squared;
    return WS3D_OK;
}

ws3d_status ws3d_halo_attach(ws3d_ctx* c, const ws3d_halo_handles* lo, const ws3d_halo_handles* hi) {
    WS3D_NOT_RESIDENT(c);
    if (!c) return WS3D_EINVAL;
    NvtxRange nv("ws3d.connect.attach", kNvtxSync);
    if (c->halo) return fail(c, WS3D_EPEER, "halo_attach: neighbours already attached");
    if (lo && (!same_geometry(c, lo->width, lo->height, lo->depth, lo->pitch) || lo->z_end != c->z0))
        return fail(c, WS3D_EINVAL, "halo_attach: lower slab [%u,%u) does not end at %u or differs in shape",
                    lo->z_begin, lo->z_end, c->z0);
    if (hi && (!same_geometry(c, hi->width, hi->height, hi->depth, hi->pitch) ||
               hi->z_begin != c->z0 + c->nz))
        return fail(c, WS3D_EINVAL, "halo_attach: upper slab [%u,%u) does not start at %u or differs in shape",
                    hi->z_begin, hi->z_end, c->z0 + c->nz);
    if ((lo && c->z0 == 0) || (hi && c->z0 + c->nz == c->Dg) || (!lo && c->z0 > 0) ||
        (!hi && c->z0 + c->nz < c->Dg))
        return fail(c, WS3D_EINVAL, "halo_attach: neighbours do not match the slab position");
    for (const ws3d_halo_handles* n : {lo, hi})
        if (n && n->ghost_planes != c->gd)
            return fail(c, WS3D_EINVAL, "halo_attach: neighbour buffers hold %u ghost planes per "
                                        "side, this slab %u", n->ghost_planes, c->gd);
    DeviceGuard g(c->desc.device);
    auto open = [&](const uint8_t* bytes, void** ptr) -> ws3d_status {
        cudaIpcMemHandle_t h;
        std::memcpy(&h, bytes, 64);
        cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) return cuda_fail(c, WS3D_EPEER, e, "cudaIpcOpenMemHandle");
        c->ipc_opened.push_back(*ptr);
        return WS3D_OK;
    };
    // one neighbour: its field buffers (plane -1 pointers), flags, c2 field
    auto map = [&](const ws3d_halo_handles* n, float** base, const float** c2,
                   unsigned long long** flag, int flag_word) -> ws3d_status {
        ws3d_status s;
        void* q = nullptr;
        const int nb = (n->caps & WS3D_HALO_CAP_TWO_STEP) ? 4 : 2;
        for (int b = 0; b < nb; ++b) {
            if ((s = open(n->buf[b], &q)) != WS3D_OK) return s;
            base[b] = static_cast<float*>(q) + (size_t)(n->ghost_planes - 1) * c->plane;
        }
        if ((s = open(n->flags, &q)) != WS3D_OK) return s;
        *flag = static_cast<unsigned long long*>(q) + flag_word;
        if (n->caps & WS3D_HALO_CAP_C2_FIELD) {
            if ((s = open(n->c2, &q)) != WS3D_OK) return s;
            *c2 = static_cast<const float*>(q);
        }
        return WS3D_OK;
    };
    ws3d_status s;
    if (lo) {  // I am its upper neighbour: I raise its flags[1]
        if ((s = map(lo, c->lo_base, &c->lo_c2, &c->lo_flag, 1)) != WS3D_OK) return s;
        c->lo_caps = lo->caps;
        c->lo_nz = lo->z_end - lo->z_begin;
        c->lo_c2u = lo->c_squared;
    }
    if (hi) {  // I am its lower neighbour: I raise its flags[0]
        if ((s = map(hi, c->hi_base, &c->hi_c2, &c->hi_flag, 0)) != WS3D_OK) return s;
        c->hi_caps = hi->caps;
        c->hi_nz = hi->z_end - hi->z_begin;
        c->hi_c2u = hi->c_squared;
    }
    c->host_ordered = false;
    return attach_common(c);
}

ws3d_status ws3d_halo_attach_local(ws3d_ctx* c, ws3d_ctx* lo, ws3d_ctx* hi) {
    WS3D_NOT_RESIDENT(c);
    if (!c) return WS3D_EINVAL;
    if (c->halo) return fail(c, WS3D_EPEER, "halo_attach_local: neighbours already attached");
    for (ws3d_ctx* n : {lo, hi}) {
        if (!n) continue;
        if (!same_geometry(c, n->W, n->H, n->Dg, n->pitch))
            return fail(c, WS3D_EINVAL, "halo_attach_local: neighbour differs in shape");
        if (n->desc.device != c->desc.device)
            return fail(c, WS3D_EINVAL,
                        "halo_attach_local: neighbours on other devices attach through "
                        "ws3d_halo_export / ws3d_halo_attach (one process per GPU)");
    }
    if ((lo && lo->z0 + lo->nz != c->z0) || (hi && hi->z0 != c->z0 + c->nz) ||
        (!lo && c->z0 > 0) || (!hi && c->z0 + c->nz < c->Dg))
        return fail(c, WS3D_EINVAL, "halo_attach_local: neighbours do not match the slab position");
    DeviceGuard g(c->desc.device);
    if (lo) {
        c->lo_caps = halo_caps(lo);  // allocates its two-step buffers when capable
        for (int b = 0; b < 4; ++b) c->lo_base[b] = lo->buf[b];
        c->lo_c2 = lo->c2f;
        c->lo_nz = lo->nz;
        c->lo_c2u = lo->desc.c_squared;
        c->lo_flag = lo->flags + 1;
    }
    if (hi) {
        c->hi_caps = halo_caps(hi);
        for (int b = 0; b < 4; ++b) c->hi_base[b] = hi->buf[b];
        c->hi_c2 = hi->c2f;
        c->hi_nz = hi->nz;
        c->hi_c2u = hi->desc.c_squared;
        c->hi_flag = hi->flags + 0;
    }
    // Same device: the slabs advance in one stream through ws3d_step_group, so
    // stream order replaces the device-side flags (two kernels that wait on one
    // another never share a GPU).
    c->host_ordered = true;
    return attach_common(c);
}

ws3d_status ws3d_halo_set_depth(ws3d_ctx* c, uint32_t depth) {
    WS3D_NOT_RESIDENT(c);
    if (!c) return WS3D_EINVAL;
    if (depth != 1 && depth != 2)
        return fail(c, WS3D_EINVAL, "halo_set_depth: depth %u is not 1 or 2", depth);
    if (!c->halo) return fail(c, WS3D_ECOMMAND, "halo_set_depth: no neighbours attached");
    DeviceGuard g(c->desc.device);
    if (depth == 2) {
        const uint32_t mine = halo_caps(c);
        const bool c2 = (mine & WS3D_HALO_CAP_C2_FIELD) != 0;
        // a neighbour fits when it is two-step capable, owns >= 2 planes, and
        // its c2 is given the same way (field, or the same uniform value)
        auto fits = [&](const float* base, uint32_t caps, uint32_t nz, float c2u) {
            return !base || ((caps & WS3D_HALO_CAP_TWO_STEP) && nz >= 2 &&
                             ((caps & WS3D_HALO_CAP_C2_FIELD) != 0) == c2 &&
                             (c2 || c2u == c->desc.c_squared));
        };
        if (!(mine & WS3D_HALO_CAP_TWO_STEP) || !fits(c->lo_base[0], c->lo_caps, c->lo_nz, c->lo_c2u) ||
            !fits(c->hi_base[0], c->hi_caps, c->hi_nz, c->hi_c2u))
            return fail(c, WS3D_EINVAL,
                        "halo_set_depth: temporal depth 2 needs this slab and its neighbours "
                        "two-step capable (auto or tma2 variant, TMA kernels, monotone sponge of "
                        "width <= 64, >= 2 planes each) with c2 given the same way");
        if (!c->peer_maps)
            return fail(c, WS3D_EPEER,
                        "halo_set_depth: tensor maps over the neighbours' buffers could not be "
                        "encoded");
    }
    c->hdepth = depth;
    c->halo_synced = false;
    c->deep_ok = false;
    ws3d_status s = rebuild_source_ghosts(c);
    return s == WS3D_OK ? rebuild_tb_sources(c) : s;
}

ws3d_status ws3d_halo_sync(ws3d_ctx* c, uint32_t phase) {
    WS3D_NOT_RESIDENT(c);
    if (!c) return WS3D_EINVAL;
    if (!c->halo) return WS3D_OK;
    if (phase > 1) return fail(c, WS3D_EINVAL, "halo_sync: phase must be 0 or 1");
    NvtxRange nv(phase == 0 ? "ws3d.connect.quiesce" : "ws3d.connect.halo_sync", kNvtxSync);
    DeviceGuard g(c->desc.device);
    // Phase 0: quiesce -- after it (and the barrier that follows on every
    // rank) no signal of an earlier step is still in flight towards anyone.
    WS3D_CUDA(c, cudaStreamSynchronize(c->stream), WS3D_EDEVICE);
    c->halo_synced = false;
    if (phase == 0) return WS3D_OK;
    // Phase 1: clear this slab's flags, then fill the neighbours' ghost planes
    // with this slab's first / last plane (two of each at temporal depth 2)
    // of the current field.
    WS3D_CUDA(c, cudaMemset(c->flags, 0, kFlagWords * sizeof(unsigned long long)), WS3D_EDEVICE);
    c->halo_steps = 0;
    const size_t P = c->plane;
    const uint32_t d = std::min(c->hdepth, c->nz);
    const size_t bytes = d * P * sizeof(float);
    float* B = c->buf[c->ip];
    if (c->lo_base[0])
        WS3D_CUDA(c, cudaMemcpyAsync(c->lo_base[c->ip] + c->lo_ghost_off, B + P, bytes,
                                     cudaMemcpyDefault, c->stream),
                  WS3D_EPEER);
    if (c->hi_base[0])
        WS3D_CUDA(c, cudaMemcpyAsync(c->hi_base[c->ip] - (d - 1) * P, B + (c->nz - d + 1) * P,
                                     bytes, cudaMemcpyDefault, c->stream),
                  WS3D_EPEER);
    WS3D_CUDA(c, cudaStreamSynchronize(c->stream), WS3D_EPEER);
    c->halo_synced = true;
    c->deep_ok = c->hdepth == 2;
    return WS3D_OK;
}

ws3d_status ws3d_step_group(ws3d_ctx* const* ctxs, uint32_t n, uint64_t steps) {
    if (!ctxs || n == 0) return WS3D_EINVAL;
    for (uint32_t k = 0; k < n; ++k) {
        ws3d_ctx* c = ctxs[k];
        if (!c) return WS3D_EINVAL;
        WS3D_NOT_RESIDENT(c);
        if (c->desc.device != ctxs[0]->desc.device || c->stream != ctxs[0]->stream)
            return fail(c, WS3D_EINVAL, "step_group: contexts must share one device and stream");
        if (c->halo && !c->halo_synced)
            return fail(c, WS3D_ECOMMAND, "step_group: fields changed since the last halo sync");
        if (c->ip != ctxs[0]->ip || c->step != ctxs[0]->step)
            return fail(c, WS3D_ECOMMAND, "step_group: contexts are at different steps");
        if (c->halo && c->hdepth == 2 && !tma_eligible(c))
            return fail(c, WS3D_ECOMMAND, "step_group: temporal depth 2 needs the TMA kernels");
    }
    DeviceGuard g(ctxs[0]->desc.device);
    for (uint64_t s = 0; s < steps;) {
        // one- or two-step launches, the same for every context
        const bool two = steps - s >= 2 && use_two_step(ctxs[0]);
        for (uint32_t k = 1; k < n; ++k)
            if (two != (steps - s >= 2 && use_two_step(ctxs[k])))
                return fail(ctxs[k], WS3D_ECOMMAND,
                            "step_group: contexts disagree on two-step launches");
        // All sources first (they touch neighbours' ghost copies), then all launches.
        for (uint32_t k = 0; k < n; ++k) {
            ws3d_status st = launch_sources(ctxs[k]);
            if (st != WS3D_OK) return st;
        }
        for (uint32_t k = 0; k < n; ++k) {
            ws3d_ctx* c = ctxs[k];
            ws3d_status st = two ? (c->c2f ? launch_tb<true>(c) : launch_tb<false>(c))
                                 : launch_step(c);
            if (st != WS3D_OK) return st;
        }
        for (uint32_t k = 0; k < n; ++k) {
            ws3d_ctx* c = ctxs[k];
            if (!two) std::swap(c->ip, c->ipp);
            c->step += two ? 2 : 1;
            c->halo_steps++;
            c->deep_ok = true;
        }
        s += two ? 2 : 1;
    }
    return WS3D_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Resident mode (host side of k_resident).
// ---------------------------------------------------------------------------
static_assert(sizeof(ws3d_resident_config) == 56, "ws3d_resident_config layout");
static_assert(sizeof(ws3d_resident_stats) == 88, "ws3d_resident_stats layout");

namespace {
template <class T>
T vload(const T* p) {
    return *reinterpret_cast<const volatile T*>(p);
}
template <class T>
void vstore(T* p, T v) {
    *reinterpret_cast<volatile T*>(p) = v;
}
bool is_pow2(uint32_t v) { return v && !(v & (v - 1)); }

// Block layout: control block | H2K header | H2K slots | K2H header | K2H slots.
size_t res_layout(uint32_t h2k_cap, uint32_t k2h_cap, size_t off[4]) {
    off[0] = sizeof(ResidentCtrl);
    off[1] = off[0] + sizeof(ResQueue);
    off[2] = off[1] + (size_t)h2k_cap * sizeof(ResMsg);
    off[3] = off[2] + sizeof(ResQueue);
    return off[3] + (size_t)k2h_cap * sizeof(ResMsg);
}

// The launch in flight (if any) has ended: take over its step count and
// buffer roles.
ws3d_status res_absorb(ws3d_ctx* c) {
    if (!c->res_alive) return WS3D_OK;
    const cudaError_t e = cudaEventQuery(c->res_done);
    if (e == cudaErrorNotReady) return WS3D_OK;
    if (e != cudaSuccess) return cuda_fail(c, WS3D_EDEVICE, e, "resident kernel");
    c->res_alive = false;
    std::atomic_thread_fence(std::memory_order_acquire);
    const uint64_t ran = vload(&c->res_ctrl->steps_run);
    const uint32_t cb = vload(&c->res_ctrl->current_buffer);
    const uint32_t why = vload(&c->res_ctrl->exit_reason);
    c->step = c->res_step0 + ran;
    if (cb & 1u) std::swap(c->ip, c->ipp);
    if (why == 1u) c->res_terminated = true;
    if (why == 3u || why == 0u) {
        c->res_terminated = true;
        const ws3d_status st = check_device_status(c);
        return st != WS3D_OK ? st
                             : fail(c, WS3D_EDEVICE, "the resident kernel left without a reason");
    }
    return WS3D_OK;
}

// Work the kernel has not consumed: queued commands, or steps while not paused.
bool res_pending(const ws3d_ctx* c) {
    if (c->res_h2k_tail != vload(&c->res_h2k->head)) return true;
    return vload(&c->res_ctrl->steps_remaining) > 0 && !vload(&c->res_ctrl->paused);
}

template <bool kC2F, bool kCells>
ws3d_status res_launch_t(ws3d_ctx* c) {
    auto kern = k_resident<kC2F, kCells, kPersTY>;
    const int threads = 32 * kPersTY;
    int per_sm = 0;
    cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, threads, 0);
    if (e != cudaSuccess || per_sm < 1) return cuda_fail(c, WS3D_ELAUNCH, e, "occupancy(resident)");
    c->res_resident = per_sm * std::max(1, c->sm_count);
    PersistentArgs q{};
    q.a = make_params(c);
    q.buf[0] = c->buf[c->ip];
    q.buf[1] = c->buf[c->ipp];
    q.bar = c->flags + kBarWord;
    // the barrier's arrival counter starts every launch at zero (stream order)
    WS3D_CUDA(c, cudaMemsetAsync(q.bar, 0, sizeof *q.bar, c->stream), WS3D_ELAUNCH);
    q.src_off = c->src_off;
    q.wavelet = c->wavelet;
    q.n_src = c->n_src;
    q.wl_len = c->wl_len;
    q.step0 = c->step;
    q.tiles_x = (c->pitch + kZsTileX - 1) / kZsTileX;
    q.tiles = q.tiles_x * ((c->H + kPersTY - 1) / kPersTY);
    const TmaSchedule sch = tma_schedule(q.tiles, c->nz, (uint32_t)c->res_resident, 4);
    q.clen = sch.clen;
    q.nitems = sch.nitems;
    if (sch.grid > c->red_blocks)
        return fail(c, WS3D_ELAUNCH, "resident grid %u above the reduction scratch (%u)", sch.grid,
                    c->red_blocks);
    ResidentArgs r{};
    r.q = q;
    char* dev = nullptr;
    e = cudaHostGetDevicePointer(reinterpret_cast<void**>(&dev), c->res_mem, 0);
    if (e != cudaSuccess) return cuda_fail(c, WS3D_EMEMORY, e, "cudaHostGetDevicePointer");
    size_t off[4];
    res_layout(c->res_cfg.h2k_capacity, c->res_cfg.k2h_capacity, off);
    r.ctrl = reinterpret_cast<ResidentCtrl*>(dev);
    r.h2k = reinterpret_cast<ResQueue*>(dev + off[0]);
    r.h2k_slots = reinterpret_cast<const ResMsg*>(dev + off[1]);
    r.k2h = reinterpret_cast<ResQueue*>(dev + off[2]);
    r.k2h_slots = reinterpret_cast<ResMsg*>(dev + off[3]);
    r.decision = reinterpret_cast<unsigned int*>(c->flags + 6);
    r.partial = c->red_scratch;
    r.progress_interval = c->res_cfg.progress_interval;
    r.idle_budget_ns = c->res_cfg.idle_budget_ns;
    r.h2k_mask = c->res_cfg.h2k_capacity - 1;
    r.k2h_capacity = c->res_cfg.k2h_capacity;
    void* args[] = {&r};
    e = cudaLaunchCooperativeKernel((const void*)kern, dim3(sch.grid), dim3(32, kPersTY, 1), args,
                                    0, c->stream);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return cuda_fail(c, WS3D_ELAUNCH, e, "cudaLaunchCooperativeKernel(k_resident)");
    }
    WS3D_CUDA(c, cudaEventRecord(c->res_done, c->stream), WS3D_EDEVICE);
    c->launches++;
    c->res_launches++;
    c->res_alive = true;
    c->res_role[0] = c->ip;
    c->res_role[1] = c->ipp;
    c->res_step0 = c->step;
    return WS3D_OK;
}

ws3d_status res_launch(ws3d_ctx* c) {
    // a stale give-up bit would make every grid barrier of the new launch fail
    unsigned int st = 0;
    WS3D_CUDA(c, cudaMemcpy(&st, c->flags + 2, sizeof st, cudaMemcpyDeviceToHost), WS3D_EDEVICE);
    if (st) return check_device_status(c);
    ResidentCtrl* k = c->res_ctrl;
    vstore(&k->has_terminated, 0u);
    vstore(&k->exit_reason, 0u);
    vstore(&k->current_buffer, 0u);
    vstore(&k->steps_run, (uint64_t)0);
    vstore(&k->current_step, c->step);
    std::atomic_thread_fence(std::memory_order_seq_cst);
    const bool f = c->c2f != nullptr, cells = !c->cells_default;
    if (f && cells) return res_launch_t<true, true>(c);
    if (f) return res_launch_t<true, false>(c);
    if (cells) return res_launch_t<false, true>(c);
    return res_launch_t<false, false>(c);
}

// Take over a finished launch; relaunch when work is waiting.
ws3d_status res_service(ws3d_ctx* c) {
    ws3d_status s = res_absorb(c);
    if (s != WS3D_OK) return s;
    if (!c->res_alive && c->res_active && !c->res_terminated && res_pending(c)) return res_launch(c);
    return WS3D_OK;
}

ws3d_status res_enqueue(ws3d_ctx* c, const ws3d_h2k_msg& m) {
    static_assert(sizeof(ws3d_h2k_msg) == sizeof(ResMsg), "H2K message size");
    const uint64_t head = vload(&c->res_h2k->head);
    if (c->res_h2k_tail - head >= c->res_cfg.h2k_capacity)
        return fail(c, WS3D_ECOMMAND, "resident: H2K queue full (%u commands not yet consumed)",
                    c->res_cfg.h2k_capacity);
    std::memcpy(&c->res_h2k_slots[c->res_h2k_tail & (c->res_cfg.h2k_capacity - 1)], &m, sizeof m);
    std::atomic_thread_fence(std::memory_order_seq_cst);  // slot before index
    vstore(&c->res_h2k->tail, ++c->res_h2k_tail);
    return WS3D_OK;
}

void res_sleep() { std::this_thread::sleep_for(std::chrono::microseconds(20)); }
uint64_t now_ns() {
    return (uint64_t)std::chrono::duration_cast<std::chrono::nanoseconds>(
               std::chrono::steady_clock::now().time_since_epoch())
        .count();
}
}  // namespace

extern "C" {

ws3d_status ws3d_resident_start(ws3d_ctx* c, const ws3d_resident_config* cfg_in) {
    if (!c) return WS3D_EINVAL;
    if (c->res_active) return WS3D_OK;  // persistent_backend.rs:253-256
    if (c->halo) return fail(c, WS3D_EINVAL, "resident mode runs on one GPU (no z-slabs)");
    ws3d_resident_config cfg{};
    if (cfg_in) cfg = *cfg_in;
    if (!cfg.progress_interval) cfg.progress_interval = 100;
    if (!cfg.h2k_capacity) cfg.h2k_capacity = 256;
    if (!cfg.k2h_capacity) cfg.k2h_capacity = 256;
    if (!cfg.idle_budget_ns) cfg.idle_budget_ns = 1000000000ull;
    if (!is_pow2(cfg.h2k_capacity) || !is_pow2(cfg.k2h_capacity) || cfg.h2k_capacity > 65536 ||
        cfg.k2h_capacity > 65536)
        return fail(c, WS3D_EINVAL, "resident: queue capacities must be powers of two <= 65536");
    DeviceGuard g(c->desc.device);
    WS3D_CUDA(c, cudaStreamSynchronize(c->stream), WS3D_EDEVICE);
    ws3d_status s = check_device_status(c);
    if (s != WS3D_OK) return s;
    size_t off[4];
    const size_t bytes = res_layout(cfg.h2k_capacity, cfg.k2h_capacity, off);
    if (c->res_mem && bytes != c->res_bytes) {
        cudaFreeHost(c->res_mem);
        c->res_mem = nullptr;
    }
    if (!c->res_mem) {
        WS3D_CUDA(c, cudaHostAlloc(&c->res_mem, bytes, cudaHostAllocMapped | cudaHostAllocPortable),
                  WS3D_EMEMORY);
        c->res_bytes = bytes;
    }
    if (!c->res_done) WS3D_CUDA(c, cudaEventCreateWithFlags(&c->res_done, cudaEventDisableTiming),
                                WS3D_EDEVICE);
    if (!c->res_side) WS3D_CUDA(c, cudaStreamCreateWithFlags(&c->res_side, cudaStreamNonBlocking),
                                WS3D_EDEVICE);
    std::memset(c->res_mem, 0, bytes);
    char* h = static_cast<char*>(c->res_mem);
    c->res_ctrl = reinterpret_cast<ResidentCtrl*>(h);
    c->res_h2k = reinterpret_cast<ResQueue*>(h + off[0]);
    c->res_h2k_slots = reinterpret_cast<ResMsg*>(h + off[1]);
    c->res_k2h = reinterpret_cast<ResQueue*>(h + off[2]);
    c->res_k2h_slots = reinterpret_cast<ResMsg*>(h + off[3]);
    c->res_h2k->capacity = cfg.h2k_capacity;
    c->res_h2k->mask = cfg.h2k_capacity - 1;
    c->res_k2h->capacity = cfg.k2h_capacity;
    c->res_k2h->mask = cfg.k2h_capacity - 1;
    c->res_ctrl->current_step = c->step;
    c->res_h2k_tail = 0;
    c->res_k2h_head = 0;
    c->res_cfg = cfg;
    c->res_terminated = false;
    c->res_active = true;
    s = res_launch(c);
    if (s != WS3D_OK) c->res_active = false;
    return s;
}

ws3d_status ws3d_resident_send(ws3d_ctx* c, const ws3d_h2k_msg* msg) {
    if (!c || !msg) return c ? fail(c, WS3D_EINVAL, "resident_send: msg is NULL") : WS3D_EINVAL;
    if (!c->res_active) return fail(c, WS3D_ECOMMAND, "resident mode is not started");
    DeviceGuard g(c->desc.device);
    ws3d_status s = res_absorb(c);
    if (s != WS3D_OK) return s;
    if (c->res_terminated)
        return fail(c, WS3D_ECOMMAND, "the resident kernel has terminated; start it again");
    if ((s = res_enqueue(c, *msg)) != WS3D_OK) return s;
    return res_service(c);
}

ws3d_status ws3d_resident_run_steps(ws3d_ctx* c, uint64_t steps) {
    ws3d_h2k_msg m{};
    m.cmd = WS3D_CMD_RUN_STEPS;
    m.param1 = steps;
    return ws3d_resident_send(c, &m);
}

ws3d_status ws3d_resident_inject_impulse(ws3d_ctx* c, uint32_t x, uint32_t y, uint32_t z,
                                         float amplitude) {
    ws3d_h2k_msg m{};
    m.cmd = WS3D_CMD_INJECT_IMPULSE;
    m.param1 = ((uint64_t)x << 32) | y;
    m.param2 = z;
    m.param4 = amplitude;
    return ws3d_resident_send(c, &m);
}

ws3d_status ws3d_resident_wait_step(ws3d_ctx* c, uint64_t step, uint64_t timeout_ns) {
    if (!c) return WS3D_EINVAL;
    if (!c->res_active) return fail(c, WS3D_ECOMMAND, "resident mode is not started");
    DeviceGuard g(c->desc.device);
    const uint64_t deadline = now_ns() + (timeout_ns ? timeout_ns : 10000000000ull);
    for (;;) {
        ws3d_status s = res_service(c);
        if (s != WS3D_OK) return s;
        const uint64_t cur = c->res_alive ? vload(&c->res_ctrl->current_step) : c->step;
        if (cur >= step) return WS3D_OK;
        if (c->res_terminated)
            return fail(c, WS3D_ECOMMAND, "the resident kernel terminated at step %llu < %llu",
                        (unsigned long long)cur, (unsigned long long)step);
        if (!c->res_alive && !res_pending(c))
            return fail(c, WS3D_ECOMMAND,
                        "step %llu < %llu and no steps pending (paused, or too few RUN_STEPS)",
                        (unsigned long long)cur, (unsigned long long)step);
        if (now_ns() > deadline)
            return fail(c, WS3D_ETIMEOUT, "timeout waiting for step %llu (at %llu)",
                        (unsigned long long)step, (unsigned long long)cur);
        res_sleep();
    }
}

ws3d_status ws3d_resident_poll(ws3d_ctx* c, ws3d_k2h_msg* out, uint32_t max, uint32_t* n_out) {
    static_assert(sizeof(ws3d_k2h_msg) == sizeof(ResMsg), "K2H message size");
    if (!c || !n_out || (max && !out)) return c ? fail(c, WS3D_EINVAL, "resident_poll: bad arguments")
                                               : WS3D_EINVAL;
    *n_out = 0;
    if (!c->res_mem) return WS3D_OK;
    const uint64_t tail = vload(&c->res_k2h->tail);
    std::atomic_thread_fence(std::memory_order_acquire);
    uint32_t k = 0;
    while (c->res_k2h_head != tail && k < max) {
        std::memcpy(&out[k++], &c->res_k2h_slots[c->res_k2h_head & (c->res_cfg.k2h_capacity - 1)],
                    sizeof(ws3d_k2h_msg));
        ++c->res_k2h_head;
    }
    std::atomic_thread_fence(std::memory_order_seq_cst);
    vstore(&c->res_k2h->head, c->res_k2h_head);
    *n_out = k;
    return WS3D_OK;
}

ws3d_status ws3d_resident_stats_get(const ws3d_ctx* c, ws3d_resident_stats* o) {
    if (!c || !o) return WS3D_EINVAL;
    std::memset(o, 0, sizeof *o);
    o->current_step = c->step;
    o->launches = c->res_launches;
    o->is_running = c->res_active;
    o->has_terminated = c->res_terminated;
    if (!c->res_ctrl) return WS3D_OK;
    const ResidentCtrl* k = c->res_ctrl;
    const bool alive = c->res_alive && cudaEventQuery(c->res_done) == cudaErrorNotReady;
    if (c->res_alive) o->current_step = vload(&k->current_step);
    o->steps_remaining = vload(&k->steps_remaining);
    o->total_energy = vload(&k->total_energy);
    o->messages_processed = vload(&k->messages_processed);
    o->k2h_dropped = vload(&k->k2h_dropped);
    o->paused = vload(&k->paused);
    o->kernel_alive = alive;
    if (vload(&k->exit_reason) == 1u) o->has_terminated = 1;
    return WS3D_OK;
}

ws3d_status ws3d_resident_download(ws3d_ctx* c, float* p, uint64_t timeout_ns) {
    if (!c || !p) return c ? fail(c, WS3D_EINVAL, "resident_download: NULL") : WS3D_EINVAL;
    if (!c->res_active) return ws3d_download(c, p, nullptr);
    DeviceGuard g(c->desc.device);
    const uint64_t deadline = now_ns() + (timeout_ns ? timeout_ns : 10000000000ull);
    for (;;) {  // until the kernel consumed every command and ran every step
        ws3d_status s = res_service(c);
        if (s != WS3D_OK) return s;
        if (!res_pending(c)) break;
        if (now_ns() > deadline)
            return fail(c, WS3D_ETIMEOUT, "resident_download: steps still pending after the timeout");
        res_sleep();
    }
    // idle kernel (or none): the fields do not change; copy on a side stream
    const float* src = c->res_alive ? c->buf[c->res_role[vload(&c->res_ctrl->current_buffer) & 1u]]
                                    : c->buf[c->ip];
    cudaError_t e = cudaMemcpy2DAsync(p, c->W * sizeof(float), src + c->plane,
                                      c->pitch * sizeof(float), c->W * sizeof(float),
                                      (size_t)c->H * c->nz, cudaMemcpyDeviceToHost, c->res_side);
    if (e != cudaSuccess) return cuda_fail(c, WS3D_EREADBACK, e, "resident_download copy");
    WS3D_CUDA(c, cudaStreamSynchronize(c->res_side), WS3D_EREADBACK);
    return WS3D_OK;
}

ws3d_status ws3d_resident_shutdown(ws3d_ctx* c, uint64_t timeout_ns) {
    if (!c) return WS3D_EINVAL;
    if (!c->res_active) return WS3D_OK;
    DeviceGuard g(c->desc.device);
    const uint64_t deadline = now_ns() + (timeout_ns ? timeout_ns : 10000000000ull);
    ws3d_status s = res_absorb(c);
    if (s == WS3D_OK && !c->res_terminated) {
        // TERMINATE also reaches a kernel that left after its idle budget: it
        // is relaunched to run the commands still queued, report the final
        // energy and post TERMINATED (persistent_fdtd.rs:942-978)
        ws3d_h2k_msg m{};
        m.cmd = WS3D_CMD_TERMINATE;
        while (res_enqueue(c, m) != WS3D_OK) {  // full queue: the kernel drains it every step
            if ((s = res_service(c)) != WS3D_OK) break;
            if (now_ns() > deadline)
                return fail(c, WS3D_ETIMEOUT, "resident_shutdown: H2K queue stays full");
            res_sleep();
        }
        c->err.clear();
        if (s == WS3D_OK) s = res_service(c);
        while (s == WS3D_OK && c->res_alive) {
            if ((s = res_absorb(c)) != WS3D_OK || !c->res_alive) break;
            if (now_ns() > deadline)
                return fail(c, WS3D_ETIMEOUT, "resident_shutdown: kernel still running after the "
                                              "timeout");
            res_sleep();
        }
    }
    c->res_active = false;
    WS3D_CUDA(c, cudaStreamSynchronize(c->stream), WS3D_EDEVICE);
    if (s != WS3D_OK && s != WS3D_ECOMMAND) return s;
    return check_device_status(c);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Volume rendering (ws3d_volume.cuh).
// ---------------------------------------------------------------------------
extern "C" {

void ws3d_volume_params_init(ws3d_volume_params* p, uint32_t width, uint32_t height) {
    if (!p) return;
    std::memset(p, 0, sizeof *p);
    p->width = width;
    p->height = height;
    p->density_scale = 2.0f;  // volume.rs:180-190
    p->step_size = 0.05f;
    p->max_steps = 256;
    p->threshold = 0.01f;
    p->cell_size = 1.0f;
    p->fov_y = 0.785398163397448309616f;  // FRAC_PI_4 (camera.rs:32)
    p->up[1] = 1.0f;
    p->default_camera = 1;
}

ws3d_status ws3d_render_volume(ws3d_ctx* c, const ws3d_volume_params* prm, float* rgba) {
    WS3D_NOT_RESIDENT(c);
    if (!c) return WS3D_EINVAL;
    if (!prm || !rgba) return fail(c, WS3D_EINVAL, "render_volume: NULL argument");
    if (prm->width == 0 || prm->height == 0 || prm->width > 16384 || prm->height > 16384 ||
        !(prm->step_size > 0.0f) || !(prm->cell_size > 0.0f) || prm->max_steps > (1u << 20) ||
        !(prm->fov_y > 0.0f && prm->fov_y < 3.1f))
        return fail(c, WS3D_EINVAL, "render_volume: bad parameters");
    if (c->nz != c->Dg)
        return fail(c, WS3D_EINVAL, "render_volume needs the whole grid on this context");
    DeviceGuard g(c->desc.device);
    ws3d_status s;
    const size_t n = (size_t)c->W * c->H * c->Dg;
    if (c->vol_elems != n) {
        dfree(c, c->vol16, c->vol_elems);
        c->vol_elems = 0;
        if ((s = dalloc(c, &c->vol16, n, "volume (f16)")) != WS3D_OK) return s;
        c->vol_elems = n;
    }
    const size_t npix = (size_t)prm->width * prm->height;
    if (c->img_elems != npix) {
        dfree(c, c->img, c->img_elems);
        c->img_elems = 0;
        if ((s = dalloc(c, &c->img, npix, "volume image")) != WS3D_OK) return s;
        c->img_elems = npix;
    }
    // update_volume (volume.rs:396-420): max |p| on the device, then p / max as f16
    const uint64_t rows = (uint64_t)c->nz * c->H;
    float* part = reinterpret_cast<float*>(c->red_scratch);
    float* mx = reinterpret_cast<float*>(c->red_scratch + c->red_blocks);
    k_maxabs_partials<<<c->red_blocks, kRedThreads, 0, c->stream>>>(owned0(c, c->buf[c->ip]), c->W,
                                                                     c->pitch, rows, part);
    if ((s = check_launch(c, "k_maxabs_partials")) != WS3D_OK) return s;
    k_fold_max<<<1, kRedThreads, 0, c->stream>>>(part, c->red_blocks, mx);
    if ((s = check_launch(c, "k_fold_max")) != WS3D_OK) return s;
    k_volume_normalize<<<c->red_blocks, 256, 0, c->stream>>>(owned0(c, c->buf[c->ip]), c->W, c->H,
                                                             c->Dg, c->pitch, c->plane, mx,
                                                             c->vol16);
    if ((s = check_launch(c, "k_volume_normalize")) != WS3D_OK) return s;

    // camera (camera.rs:51-61 for_grid, :98-110 look_at_rh / perspective_rh),
    // f32 operations in this order (the CPU restatement repeats them)
    VolumeArgs v{};
    v.vol = c->vol16;
    v.W = c->W;
    v.H = c->H;
    v.D = c->Dg;
    v.gx = (float)c->W * prm->cell_size;
    v.gy = (float)c->H * prm->cell_size;
    v.gz = (float)c->Dg * prm->cell_size;
    float eye[3], tgt[3];
    if (prm->default_camera) {
        const float cx = v.gx / 2.0f, cy = v.gy / 2.0f, cz = v.gz / 2.0f;
        const float dist = std::max(std::max(v.gx, v.gz) * 1.5f, 5.0f);
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
    float len = std::sqrt(f[0] * f[0] + f[1] * f[1] + f[2] * f[2]);
    if (!(len > 0.0f)) return fail(c, WS3D_EINVAL, "render_volume: eye == target");
    for (float& q : f) q = q / len;
    const float* up = prm->up;
    float r[3] = {f[1] * up[2] - f[2] * up[1], f[2] * up[0] - f[0] * up[2],
                  f[0] * up[1] - f[1] * up[0]};
    len = std::sqrt(r[0] * r[0] + r[1] * r[1] + r[2] * r[2]);
    if (!(len > 0.0f)) return fail(c, WS3D_EINVAL, "render_volume: up is parallel to the view");
    for (float& q : r) q = q / len;
    const float u[3] = {r[1] * f[2] - r[2] * f[1], r[2] * f[0] - r[0] * f[2],
                        r[0] * f[1] - r[1] * f[0]};
    for (int k = 0; k < 3; ++k) {
        v.eye[k] = eye[k];
        v.fwd[k] = f[k];
        v.right[k] = r[k];
        v.upv[k] = u[k];
    }
    v.tan_half = (float)std::tan((double)prm->fov_y * 0.5);
    v.aspect = (float)prm->width / (float)prm->height;
    v.density_scale = prm->density_scale;
    v.step_size = prm->step_size;
    v.threshold = prm->threshold;
    v.max_steps = prm->max_steps;
    v.width = prm->width;
    v.height = prm->height;
    for (int k = 0; k < 4; ++k) v.bg[k] = prm->background[k];
    v.composite = prm->composite;
    v.out = c->img;
    const dim3 blk(16, 16), grd((prm->width + 15) / 16, (prm->height + 15) / 16);
    k_volume_render<<<grd, blk, 0, c->stream>>>(v);
    if ((s = check_launch(c, "k_volume_render")) != WS3D_OK) return s;
    WS3D_CUDA(c, cudaMemcpyAsync(rgba, c->img, npix * sizeof(float4), cudaMemcpyDeviceToHost,
                                 c->stream),
              WS3D_EREADBACK);
    WS3D_CUDA(c, cudaStreamSynchronize(c->stream), WS3D_EREADBACK);
    return WS3D_OK;
}

}  // extern "C"
