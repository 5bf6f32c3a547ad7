/*
 * ws3d.h -- C-ABI of the B200-native WaveSim3D FDTD step library (libws3d.so).
 *
 * This is the drop-in boundary for the ringkernel-wavesim3d GPU backends of
 * mivertowski/RustCompute.  Each entry point names the reference interface it
 * replaces (paths relative to crates/ringkernel-wavesim3d/ unless stated).
 *
 * Conventions
 *  - Plain C types only: an opaque context handle, pointers and sizes.
 *  - Every function returns a ws3d_status (no exceptions cross the ABI).  On
 *    failure ws3d_last_error(ctx) holds a one-line message.  The status codes
 *    map 1:1 onto the reference's error enums GpuError (gpu_backend.rs:13-23)
 *    and PersistentBackendError (persistent_backend.rs:58-84).
 *  - Host field buffers are caller-owned, contiguous, z-major f32 arrays:
 *    index = z*W*H + y*W + x (grid3d.rs:120-122), covering the planes the
 *    context owns (the whole grid unless a z-slab was requested).
 *  - Device buffers are owned by the context and freed by ws3d_destroy.
 *  - Launches are asynchronous on the context's stream; calls that return host
 *    data (download, energy, max) synchronise that stream.
 *  - One context per host thread.  There is no CPU fallback: when the device,
 *    the kernel image or a launch fails, the call fails.
 *
 * Semantics of one step (grid3d.rs:222-269, gpu_backend.rs:27-100):
 *   interior Normal cell:  lap   = ((((W+E)+S)+N)+D)+U - 6p
 *                          p_new = (2p - p_prev) + c2*lap
 *                          out   = p_new*damping [*sponge(d)]
 *   any other cell:        out   = p_prev
 *   Absorber/Obstacle:     out  *= reflection_coeff
 *   then (pressure, pressure_prev) = (out, pressure)
 * every multiply and add separately rounded (no FMA), so results are
 * bit-identical to the reference CPU arithmetic.
 */
#ifndef WS3D_H
#define WS3D_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define WS3D_ABI_VERSION 1u

#if defined(__GNUC__)
#define WS3D_API __attribute__((visibility("default")))
#else
#define WS3D_API
#endif

typedef enum ws3d_status {
    WS3D_OK = 0,
    WS3D_EDEVICE = 1,     /* GpuError::DeviceError, PersistentBackendError::DeviceError */
    WS3D_ECOMPILE = 2,    /* GpuError::CompileError (no kernel image for this device) */
    WS3D_ELAUNCH = 3,     /* GpuError::LaunchError, PersistentBackendError::LaunchError */
    WS3D_EMEMORY = 4,     /* GpuError::MemoryError */
    WS3D_ESIMULATION = 5, /* PersistentBackendError::SimulationError */
    WS3D_ECOMMAND = 6,    /* PersistentBackendError::CommandError */
    WS3D_EREADBACK = 7,   /* PersistentBackendError::ReadbackError */
    WS3D_EINVAL = 8,      /* invalid argument: size, index, null pointer */
    WS3D_ETIMEOUT = 9,    /* a device-side bounded wait gave up */
    WS3D_EPEER = 10       /* peer access or neighbour attach failed */
} ws3d_status;

/* Step-kernel variants (all run on the GPU; none falls back to the CPU). */
enum {
    WS3D_VARIANT_AUTO = 0,     /* default: on one GPU with the default face layout and
                                  W > 128, H >= 16 the two-step kernel of TMA2 where it
                                  applies, else single TMA steps; ZSTREAM otherwise
                                  (z-slabs, cell arrays, narrow grids; NAIVE for
                                  narrow one-GPU grids of at most 8 MiB a field), except that
                                  ws3d_step(n >= 2) on a small one-GPU grid (rows of at
                                  most 128 cells, default faces) is one persistent launch
                                  with the field in shared memory */
    WS3D_VARIANT_ZSTREAM = 1,  /* 2-D tile streaming along z, 128-bit loads, register
                                  prefetch; the kernel used for z-slabs and cell arrays */
    WS3D_VARIANT_NAIVE = 2,    /* one thread per cell, fused boundary (comparator) */
    WS3D_VARIANT_REFSHAPE = 3, /* the reference's launch shape: 8x8x4 stencil launch
                                  plus a separate full-grid boundary launch (comparator) */
    WS3D_VARIANT_TMA = 4,      /* persistent, TMA-fed 4-stage shared-memory pipeline (one GPU) */
    WS3D_VARIANT_ASYNC = 5,    /* persistent, cp.async-fed 4-stage pipeline (one GPU or z-slabs) */
    WS3D_VARIANT_TMA2 = 6      /* two steps per launch (temporal blocking), TMA-fed, one GPU,
                                  default face layout, <= 32 sources; allocates two more
                                  field buffers on first use; an odd last step and contexts
                                  it cannot serve run single TMA steps */
};

typedef struct ws3d_desc {
    uint32_t width, height, depth; /* global grid in cells (GridParams, grid3d.rs:486-500) */
    float c_squared;               /* scalar Courant^2 (AcousticParams3D::c_squared) */
    float damping;                 /* AcousticParams3D::simple_damping */
    uint32_t sponge_width;         /* sponge width in cells, 0 = off */
    float sponge_max;              /* sponge coefficient at the face */
    int32_t device;                /* CUDA device ordinal */
    uint32_t z_begin, z_end;       /* owned global z planes [z_begin, z_end); 0,0 = all */
    uint32_t variant;              /* WS3D_VARIANT_* */
    uint32_t reserved0;
    uint64_t spin_budget;          /* bounded-wait iterations for device waits, 0 = default */
} ws3d_desc;

typedef struct ws3d_stats {
    uint64_t step;                 /* steps taken since create/reset (grid.step) */
    uint64_t kernel_launches;      /* kernels this context launched since create */
    uint64_t device_bytes;         /* device memory held by the context */
    uint32_t width, height, depth; /* global grid */
    uint32_t z_begin, z_end;       /* owned planes */
    uint32_t pitch;                /* device row pitch in floats (multiple of 32) */
    uint32_t variant;
    uint32_t has_c2_field;
    uint32_t has_cell_field;
    uint32_t n_sources;
    uint32_t two_step_launches;    /* two-step (temporally blocked) launches since create,
                                      saturating at 2^32 - 1 */
} ws3d_stats;

typedef struct ws3d_ctx ws3d_ctx;

/* Library identification. */
WS3D_API uint32_t ws3d_abi_version(void);
WS3D_API const char *ws3d_status_string(ws3d_status s);

/* Fill `d` with defaults for a W x H x D grid: c_squared 0.25, damping 1,
 * no sponge, device 0, whole grid, default variant. */
WS3D_API void ws3d_desc_init(ws3d_desc *d, uint32_t width, uint32_t height, uint32_t depth);

/* GpuBackend3D::new (gpu_backend.rs:204-311): allocate device state for the
 * grid and set up the reference boundary layout (grid3d.rs:96-116: every face
 * cell Absorber with reflection 0.1, every other cell Normal).  Fields start at
 * zero; upload them with ws3d_upload. */
WS3D_API ws3d_status ws3d_create(const ws3d_desc *desc, ws3d_ctx **out);

/* Drop for GpuBackend3D: free every device buffer. NULL is accepted. */
WS3D_API void ws3d_destroy(ws3d_ctx *ctx);

/* One-line message of the last failure on `ctx` ("" when none). */
WS3D_API const char *ws3d_last_error(const ws3d_ctx *ctx);

/* GpuBackend3D::upload_pressure (gpu_backend.rs:391-401): copy pressure and
 * pressure_prev from the host.  Either pointer may be NULL to leave it. */
WS3D_API ws3d_status ws3d_upload(ws3d_ctx *ctx, const float *pressure, const float *pressure_prev);

/* GpuBackend3D::download_pressure (gpu_backend.rs:383-388): copy the current
 * field (and, when non-NULL, the previous field) to the host.  Synchronous. */
WS3D_API ws3d_status ws3d_download(ws3d_ctx *ctx, float *pressure, float *pressure_prev);

/* Set the step counter (SimulationGrid3D::step, grid3d.rs:57), which indexes
 * the source wavelets; used to resume from a checkpoint
 * (ringkernel-core checkpoint.rs CheckpointMetadata::current_step). */
WS3D_API ws3d_status ws3d_set_step(ws3d_ctx *ctx, uint64_t step);

/* GpuBackend3D::reset (gpu_backend.rs:404-408): upload both fields and set the
 * step counter to zero. */
WS3D_API ws3d_status ws3d_reset(ws3d_ctx *ctx, const float *pressure, const float *pressure_prev);

/* Upload SimulationGrid3D::cell_types (u8: 0 Normal, 1 Absorber, 2 Reflector,
 * 3 Obstacle, gpu_backend.rs:261-270) and reflection_coeff, as
 * GpuBackend3D::new does (gpu_backend.rs:260-292).  Passing NULL for both
 * returns to the default face layout, which the kernels evaluate without
 * reading any per-cell boundary data. */
WS3D_API ws3d_status ws3d_set_cells(ws3d_ctx *ctx, const uint8_t *cell_types, const float *reflection);

/* Per-cell Courant^2 field (north-star extension of the scalar c_squared,
 * grid3d.rs:223).  NULL returns to the scalar desc.c_squared. */
WS3D_API ws3d_status ws3d_set_c2_field(ws3d_ctx *ctx, const float *c2);

/* Point sources driven every step with the inject_impulse semantic
 * (grid3d.rs:146-152; per-step drive as in bin/wavesim3d.rs:80-100): before
 * step s, for k in 0..n: a = s < len ? wavelet[k*len + s] : 0,
 * pressure[i_k] += a, pressure_prev[i_k] += a*0.5.  xyz holds n global (x,y,z)
 * triples.  n = 0 removes all sources. */
WS3D_API ws3d_status ws3d_set_sources(ws3d_ctx *ctx, uint32_t n, const uint32_t *xyz,
                             const float *wavelet, uint64_t len);

/* GpuBackend3D::step (gpu_backend.rs:314-380), n times.  Asynchronous.  With
 * the auto variant the library picks the launches: pairs of steps of wide
 * grids go to the two-step kernel, and n >= 2 steps of a small one-GPU grid
 * (rows of at most 128 cells, default faces, field within the SMs' shared
 * memory) to one persistent launch; the fields are bit-identical to single
 * steps either way. */
WS3D_API ws3d_status ws3d_step(ws3d_ctx *ctx, uint64_t n);

/* ws3d_step plus CUDA-event timing of every step-kernel launch on the
 * context's stream; synchronises and returns the summed kernel time in ms
 * (benchmark support: bin/benchmark.rs:75-77 times step_n on the host
 * without a synchronise, this measures on the device).  n <= 2^20.  The
 * events form a ring of 256 pairs: when the host gets 256 launches ahead it
 * waits for the oldest one before reusing its pair. */
WS3D_API ws3d_status ws3d_step_timed(ws3d_ctx *ctx, uint64_t n, double *kernel_ms);

/* ws3d_step_timed in two halves, so that a caller can record its own event
 * right behind the last launch: _begin enqueues the n steps with their event
 * pairs and returns without synchronising; _end synchronises, returns the
 * summed kernel time of the launches since _begin and reports device-side
 * errors.  (No counterpart in the reference: benchmark support.) */
WS3D_API ws3d_status ws3d_step_timed_begin(ws3d_ctx *ctx, uint64_t n);
WS3D_API ws3d_status ws3d_step_timed_end(ws3d_ctx *ctx, double *kernel_ms);

/* z-slab diagnostics: device nanoseconds this slab's step kernels spent in
 * neighbour-flag waits that did not pass at once, and how many such waits
 * there were, summed since the last reset (ws3d_halo_sync also clears them).
 * reset != 0 clears both after reading.  Synchronises the context's stream.
 * The reference has no device-side waits to account (its multi-GPU runtime
 * synchronises on the host, ringkernel-cuda multi_gpu/runtime.rs:782-870). */
WS3D_API ws3d_status ws3d_halo_wait_stats(ws3d_ctx *ctx, uint64_t *wait_ns, uint64_t *waits,
                                          int reset);

/* PersistentBackend::step (persistent_backend.rs:269-336): n steps inside ONE
 * cooperative launch (the reference's persistent kernel, generated by
 * ringkernel-cuda-codegen persistent_fdtd.rs:713-978).  All CTAs are
 * co-resident and meet at a bounded software grid barrier after each step
 * (two barriers when point sources are set).  Asynchronous; ws3d_sync reports
 * WS3D_ETIMEOUT if a barrier or neighbour wait gave up.  Same results, bit for
 * bit, as ws3d_step(ctx, n); works on z-slabs (ws3d_halo_attach) too. */
WS3D_API ws3d_status ws3d_step_persistent(ws3d_ctx *ctx, uint64_t n);

/* GpuBackend3D::inject_impulse (gpu_backend.rs:411-442). Out-of-range
 * coordinates are ignored like grid3d.rs:147. */
WS3D_API ws3d_status ws3d_inject_impulse(ws3d_ctx *ctx, uint32_t x, uint32_t y, uint32_t z,
                                float amplitude);

/* GpuBackend3D::inject_spherical_impulse (gpu_backend.rs:445-487), with the
 * CPU semantics of grid3d.rs:161-191: factor = expf(-d2/(2r)) for d2 <= r^2,
 * pressure += a*factor, pressure_prev += a*factor*0.5.  The factors are
 * evaluated on the host in f32 and applied by a kernel. */
WS3D_API ws3d_status ws3d_inject_spherical_impulse(ws3d_ctx *ctx, uint32_t cx, uint32_t cy,
                                          uint32_t cz, float amplitude, float radius);

/* SimulationGrid3D::total_energy (grid3d.rs:445-447), accumulated in f64 on
 * the device over the owned cells.  Synchronous. */
WS3D_API ws3d_status ws3d_energy(ws3d_ctx *ctx, double *sum_sq);

/* Energy (sum of p^2, accumulated in f64) of a caller-owned device field,
 * for callers that cannot allocate device memory when they need it: real-time
 * loops (an audio callback sampling the field) that must not block on the
 * device synchronisation cudaMalloc/cudaFree can imply, and host applications
 * that own all device memory through their own pool and forbid libraries from
 * allocating.  No counterpart in the reference.
 *
 * field:  device pointer, nz planes of height rows, row pitch `pitch` floats
 *         (pitch >= width; pitch == width for a dense z-major array).
 * result: device pointer to one double, written by the call.
 * stream: cudaStream_t to launch on (NULL = the legacy default stream).
 * errbuf: optional buffer for a one-line message on failure.
 * Runs on the calling thread's current device, allocates nothing and
 * returns without synchronising.  Its scratch is a fixed array of
 * WS3D_STATIC_ENERGY_MAX_PLANES doubles (one per plane, 64 KiB) that every
 * GPU loading this library holds until exit; nz above that limit is
 * rejected with WS3D_EINVAL.  The first call on a device resolves the
 * array's device address (set-up, once per device): make that first call
 * before any stream capture.  The address stays cached, so calls after a
 * cudaDeviceReset of that device are not supported.  A CUDA error that is
 * already pending when the call starts is reported (WS3D_ELAUNCH) and left
 * pending; nothing is launched then.
 * All calls on a device share the array, so calls that overlap on the GPU
 * (different streams, no ordering between them) race; each call writes every
 * entry it reads, so nothing carries over from an earlier call. */
#define WS3D_STATIC_ENERGY_MAX_PLANES 8192u
WS3D_API ws3d_status ws3d_field_energy_static(const float *field, uint32_t width,
                                              uint32_t height, uint32_t nz, uint32_t pitch,
                                              double *result, void *stream, char *errbuf,
                                              size_t errlen);

/* SimulationGrid3D::max_pressure (grid3d.rs:450-455).  Synchronous. */
WS3D_API ws3d_status ws3d_max_pressure(ws3d_ctx *ctx, float *max_abs);

/* SimulationGrid3D::get_xy_slice / get_xz_slice / get_yz_slice
 * (grid3d.rs:413-442) read straight from the device field.  axis 0: XY plane
 * at z = index (W*H floats); 1: XZ at y = index (W*nz floats, owned planes);
 * 2: YZ at x = index (H*nz floats, owned planes).  index is clamped to the
 * grid like the reference.  Synchronous. */
WS3D_API ws3d_status ws3d_get_slice(ws3d_ctx *ctx, uint32_t axis, uint32_t index, float *out);

/* SimulationGrid3D::sample_pressure (grid3d.rs:373-411): trilinear samples
 * of the current field at n positions (x, y, z triples in metres, cells of
 * `cell_size` metres), f32 in the reference order, for the binaural
 * microphone and other probes.  Positions must lie in the grid (and, on a
 * z-slab, between its own planes).  Synchronous. */
WS3D_API ws3d_status ws3d_sample_pressure(ws3d_ctx *ctx, uint32_t n, const float *pos_m,
                                          float cell_size, float *out);

/* GpuBackend3D::memory_usage (gpu_backend.rs:490-493): device bytes held. */
WS3D_API size_t ws3d_memory_usage(const ws3d_ctx *ctx);

/* Wait for every launch on the context's stream.  Returns WS3D_ETIMEOUT
 * when a bounded device wait of the z-slab exchange gave up since the last
 * check (the status is cleared by reporting it). */
WS3D_API ws3d_status ws3d_sync(ws3d_ctx *ctx);

/* Use a caller-owned cudaStream_t (passed as void*) for every later launch;
 * NULL returns to the context's own stream (the stream in use is synchronised
 * first, so it must still be alive).  ws3d_destroy never touches a caller's
 * stream: with one set, it synchronises the device instead. */
WS3D_API ws3d_status ws3d_set_stream(ws3d_ctx *ctx, void *cuda_stream);
WS3D_API ws3d_status ws3d_get_stream(const ws3d_ctx *ctx, void **cuda_stream);

WS3D_API ws3d_status ws3d_stats_get(const ws3d_ctx *ctx, ws3d_stats *out);

/* ---------------------------------------------------------------------------
 * z-slab decomposition over several GPUs (one process per GPU).
 *
 * The reference has no multi-GPU FDTD; the exchange follows its P2P
 * primitives (crates/ringkernel-cuda/src/multi_gpu/runtime.rs:377-434 peer
 * enable, :782-870 cuMemcpyPeerAsync) but moves the halo inside the step
 * kernel: the CTAs that compute a slab's first / last plane also store it
 * into the neighbour's ghost plane over NVLink; a one-thread kernel then
 * raises the neighbour's step-stamped flag (release, system scope); the
 * neighbour's boundary CTAs wait for it (acquire, bounded) while its
 * interior CTAs run.  Results are bit-identical to one GPU.
 *
 * Protocol (every rank, same order):
 *   create with desc.z_begin/z_end -> upload -> ws3d_halo_export -> exchange
 *   the handles (e.g. all_gather) -> ws3d_halo_attach(lower, upper) ->
 *   [ws3d_halo_set_depth(2) when every rank's export has WS3D_HALO_CAP_TWO_STEP]
 *   -> ws3d_halo_sync(0) -> barrier -> ws3d_halo_sync(1) -> barrier -> steps.
 * After any upload/reset, repeat the two ws3d_halo_sync phases.
 *
 * Temporal depth 2 (two steps per exchange): the field buffers of a z-slab
 * carry two ghost planes per side.  Each pair of steps runs k_step_tma2,
 * which also computes p_{t+1} on the first ghost plane of each side (from two
 * ghost planes of p_t and the neighbour's own p_{t-1} and c2 plane, read over
 * NVLink) and stores p_{t+2} of its two first / last planes into the
 * neighbours' ghost planes; single steps (odd counts) store two planes too.
 * Every rank takes the same sequence of one- and two-step launches (the
 * choice depends only on the step count and on state all ranks share), so
 * the buffer roles stay aligned across ranks.
 * ------------------------------------------------------------------------- */
#define WS3D_HALO_CAP_TWO_STEP 1u  /* four field buffers exported, two-step capable */
#define WS3D_HALO_CAP_C2_FIELD 2u  /* a c2 field is exported */

typedef struct ws3d_halo_handles {
    uint8_t buf[4][64];   /* cudaIpcMemHandle_t of the field buffers (2, 3: two-step capable) */
    uint8_t flags[64];    /* cudaIpcMemHandle_t of the flag block */
    uint8_t c2[64];       /* cudaIpcMemHandle_t of the c2 field (WS3D_HALO_CAP_C2_FIELD) */
    uint32_t width, height, depth, pitch;
    uint32_t z_begin, z_end;
    int32_t device;
    uint32_t caps;        /* WS3D_HALO_CAP_* */
    uint32_t ghost_planes;  /* ghost planes per side in the field buffers */
    float c_squared;      /* the slab's uniform c2 (desc.c_squared) */
} ws3d_halo_handles;

/* Export this slab's buffers and flags for its neighbours. */
WS3D_API ws3d_status ws3d_halo_export(ws3d_ctx *ctx, ws3d_halo_handles *out);

/* Map the neighbours' exports (NULL at a global z face).  Fails with
 * WS3D_EPEER when a mapping cannot be opened, WS3D_EINVAL when the slabs are
 * not adjacent or differ in shape. */
WS3D_API ws3d_status ws3d_halo_attach(ws3d_ctx *ctx, const ws3d_halo_handles *lower,
                                      const ws3d_halo_handles *upper);

/* In-process neighbours on the same device (tests and single-GPU slab
 * splits): no device-side waits; advance them together with ws3d_step_group
 * on one shared stream. */
WS3D_API ws3d_status ws3d_halo_attach_local(ws3d_ctx *ctx, ws3d_ctx *lower, ws3d_ctx *upper);

/* Steps per exchange after attach: 1 (default) or 2 (temporal blocking).  2
 * needs this slab and both neighbours to be two-step capable, at least two
 * owned planes on each, and the same c2-field presence; every rank of the
 * decomposition must set the same depth (decide it from all ranks' exports).
 * Fails with WS3D_EINVAL otherwise.  Call before ws3d_halo_sync. */
WS3D_API ws3d_status ws3d_halo_set_depth(ws3d_ctx *ctx, uint32_t depth);

/* Phase 0: wait for this slab's stream (no signal of an earlier step stays in
 * flight).  Phase 1: clear this slab's flags, copy its first and last planes
 * into the neighbours' ghost planes and wait for the copies.  Run phase 0 on
 * every rank, barrier, phase 1 on every rank, barrier. */
WS3D_API ws3d_status ws3d_halo_sync(ws3d_ctx *ctx, uint32_t phase);

/* Advance same-device slab contexts (ws3d_halo_attach_local) in lockstep:
 * per step, every context's sources, then every context's step kernel, all
 * on their shared stream. */
WS3D_API ws3d_status ws3d_step_group(ws3d_ctx *const *ctxs, uint32_t n, uint64_t steps);

/* ---------------------------------------------------------------------------
 * Resident (command-driven) persistent kernel, one GPU.
 *
 * The reference's persistent backend (persistent_backend.rs:174-446 over
 * ringkernel-cuda persistent.rs:571-1050, kernel persistent_fdtd.rs:713-978)
 * keeps one kernel running and drives it through queues in pinned mapped
 * host memory: host-to-kernel commands (H2K) and kernel-to-host responses
 * (K2H), 64-byte messages with the reference host's layout and codes
 * (ringkernel-cuda persistent.rs:571-590, 807-824; codes persistent_fdtd.rs:257-271).  Here the kernel's leader thread drains the
 * H2K queue between steps; all CTAs meet at a bounded grid barrier once per
 * step and run the same cell body as ws3d_step (bit-identical fields).
 * Progress (step, steps remaining, energy = sum of p^2, deterministic) goes
 * to K2H every progress_interval steps and on GET_PROGRESS.
 *
 * Differences, on purpose: INJECT_IMPULSE applies ws3d_inject_impulse's
 * semantics (p += a, p_prev += a/2), not the reference kernel's p-only add,
 * so that resident and per-step runs stay bit-identical; and an idle kernel
 * (no steps to run) does not spin forever: after idle_budget_ns without work
 * it leaves, and the next resident call that finds pending commands or steps
 * relaunches it transparently (the state lives in device memory).  While
 * resident mode is active the context accepts only ws3d_resident_* calls,
 * ws3d_stats_get, ws3d_last_error and ws3d_memory_usage; the others return
 * WS3D_ECOMMAND.  One GPU (no z-slabs).
 * ------------------------------------------------------------------------- */
enum {
    WS3D_CMD_NOP = 0,
    WS3D_CMD_RUN_STEPS = 1,      /* param1: steps to add */
    WS3D_CMD_PAUSE = 2,
    WS3D_CMD_RESUME = 3,
    WS3D_CMD_TERMINATE = 4,
    WS3D_CMD_INJECT_IMPULSE = 5, /* param1: (x << 32) | y, param2: z, param4: amplitude */
    WS3D_CMD_SET_SOURCE = 6,     /* not handled (the reference kernel ignores it): RESP_ERROR */
    WS3D_CMD_GET_PROGRESS = 7
};
enum {
    WS3D_RESP_ACK = 0,
    WS3D_RESP_PROGRESS = 1,
    WS3D_RESP_ERROR = 2,
    WS3D_RESP_TERMINATED = 3,
    WS3D_RESP_ENERGY = 4
};

typedef struct ws3d_h2k_msg { /* H2KMessage, ringkernel-cuda persistent.rs:571-590 (64 bytes) */
    uint32_t cmd;
    uint32_t flags;
    uint64_t cmd_id;
    uint64_t param1;
    uint32_t param2;
    uint32_t param3;
    float param4;
    float param5;
    uint64_t reserved[3];
} ws3d_h2k_msg;

typedef struct ws3d_k2h_msg { /* K2HMessage, ringkernel-cuda persistent.rs:807-824 (64 bytes) */
    uint32_t resp_type;
    uint32_t flags;
    uint64_t cmd_id;
    uint64_t step;
    uint64_t steps_remaining;
    float energy;
    uint32_t error_code;
    uint64_t reserved[3];
} ws3d_k2h_msg;

typedef struct ws3d_resident_config { /* PersistentBackendConfig, persistent_backend.rs:88-99 */
    uint64_t progress_interval; /* 0 = 100 */
    uint32_t h2k_capacity;      /* power of two <= 65536, 0 = 256 */
    uint32_t k2h_capacity;      /* power of two <= 65536, 0 = 256 */
    uint64_t idle_budget_ns;    /* 0 = 1 s */
    uint64_t reserved[4];
} ws3d_resident_config;

typedef struct ws3d_resident_stats { /* PersistentBackendStats, persistent_backend.rs:134-152 */
    uint64_t current_step;
    uint64_t steps_remaining;
    float total_energy;          /* at the last progress report */
    uint32_t has_terminated;     /* the kernel left after TERMINATE (or gave up) */
    uint64_t messages_processed;
    uint64_t k2h_dropped;        /* responses dropped because the K2H queue was full */
    uint64_t launches;           /* launches of the resident kernel, relaunches included */
    uint32_t is_running;         /* resident mode active (started, not shut down) */
    uint32_t kernel_alive;       /* a resident kernel occupies the GPU right now */
    uint32_t paused;
    uint32_t reserved32;
    uint64_t reserved[3];
} ws3d_resident_stats;

/* PersistentBackend::start: allocate the mapped queues (first call) and
 * launch the resident kernel on the context's stream.  cfg may be NULL. */
WS3D_API ws3d_status ws3d_resident_start(ws3d_ctx *ctx, const ws3d_resident_config *cfg);
/* Enqueue one command; WS3D_ECOMMAND when the H2K queue is full.  Relaunches
 * an idle-exited kernel. */
WS3D_API ws3d_status ws3d_resident_send(ws3d_ctx *ctx, const ws3d_h2k_msg *msg);
/* RUN_STEPS / INJECT_IMPULSE commands (PersistentSimulation::run_steps,
 * inject_impulse). */
WS3D_API ws3d_status ws3d_resident_run_steps(ws3d_ctx *ctx, uint64_t steps);
WS3D_API ws3d_status ws3d_resident_inject_impulse(ws3d_ctx *ctx, uint32_t x, uint32_t y,
                                                  uint32_t z, float amplitude);
/* Block until the kernel reports current_step >= step (PersistentBackend::step
 * polls the control block the same way, persistent_backend.rs:283-326);
 * WS3D_ETIMEOUT after timeout_ns (0 = 10 s, the reference's timeout). */
WS3D_API ws3d_status ws3d_resident_wait_step(ws3d_ctx *ctx, uint64_t step, uint64_t timeout_ns);
/* PersistentBackend::poll_responses: drain up to max K2H messages. */
WS3D_API ws3d_status ws3d_resident_poll(ws3d_ctx *ctx, ws3d_k2h_msg *out, uint32_t max,
                                        uint32_t *n_out);
/* PersistentBackend::stats (reads the mapped control block). */
WS3D_API ws3d_status ws3d_resident_stats_get(const ws3d_ctx *ctx, ws3d_resident_stats *out);
/* PersistentBackend::download_pressure: waits (bounded) until no steps are
 * pending, then copies the current field on a side stream while the kernel
 * stays resident. */
WS3D_API ws3d_status ws3d_resident_download(ws3d_ctx *ctx, float *pressure, uint64_t timeout_ns);
/* PersistentBackend::shutdown: TERMINATE, wait (bounded; 0 = 10 s) for the
 * kernel to leave, and hand the fields back to the ordinary API (step count
 * and buffer roles follow the steps the kernel ran). */
WS3D_API ws3d_status ws3d_resident_shutdown(ws3d_ctx *ctx, uint64_t timeout_ns);

/* ---------------------------------------------------------------------------
 * Headless volume ray-march of the pressure field (one context holding the
 * whole grid).  Restates the reference's volume renderer
 * (visualization/volume.rs:76-160 shader, :396-420 update_volume; camera
 * camera.rs:51-61, 98-110) without a graphics pipeline: the field is
 * normalised by max(max|p|, 0.001) and stored as f16, each pixel's primary
 * ray is marched through the box [0, grid_size] with linear filtering and
 * clamp-to-edge sampling, blue-white-red colour mapping and front-to-back
 * compositing, and RGBA floats are returned.  Every operation is a separately
 * rounded f32 operation, so the CPU restatement in oracle/ matches bit for
 * bit.
 * ------------------------------------------------------------------------- */
typedef struct ws3d_volume_params {
    uint32_t width, height;   /* image size in pixels */
    float density_scale;      /* VolumeParams::density_scale, 2.0 */
    float step_size;          /* world units per march step, 0.05 */
    uint32_t max_steps;       /* 256 */
    float threshold;          /* |p| below it is transparent, 0.01 */
    float cell_size;          /* grid_size = (W, H, D) * cell_size (world units), 1.0 */
    float fov_y;              /* radians, pi/4 */
    float eye[3];             /* camera position */
    float target[3];          /* look-at point */
    float up[3];              /* (0, 1, 0) */
    uint32_t default_camera;  /* 1: Camera3D::for_grid (camera.rs:51-61); eye and target ignored */
    float background[4];      /* target colour when composite = 1 */
    uint32_t composite;       /* 0: the fragment output (RGBA, 0 where discarded);
                                 1: BlendState::ALPHA_BLENDING over background */
    uint32_t reserved[3];
} ws3d_volume_params;

/* Defaults of VolumeParams (volume.rs:180-190) and Camera3D::for_grid. */
WS3D_API void ws3d_volume_params_init(ws3d_volume_params *p, uint32_t width, uint32_t height);
/* Render into rgba (host, width * height * 4 floats, row-major, row 0 at the
 * top).  Keeps a W x H x D f16 copy and the image buffer on the device. */
WS3D_API ws3d_status ws3d_render_volume(ws3d_ctx *ctx, const ws3d_volume_params *params,
                                        float *rgba);

#ifdef __cplusplus
}
#endif

#endif /* WS3D_H */
