// ws3d.hpp -- C++ mirror of the reference's GPU backends over the C-ABI.
//
// Header-only RAII wrappers with the method names and error behaviour of
//   GpuBackend3D      crates/ringkernel-wavesim3d/src/simulation/gpu_backend.rs:172-494
//   PersistentBackend crates/ringkernel-wavesim3d/src/simulation/persistent_backend.rs:174-446
// Errors are thrown as ws3d::GpuError carrying the ws3d_status (the
// reference returns Result<_, GpuError / PersistentBackendError>); nothing
// falls back to the CPU.  Link with -lws3d.
#pragma once

#include <cstddef>
#include <cstdint>
#include <stdexcept>
#include <string>
#include <utility>

#include "ws3d.h"

namespace ws3d {

class GpuError : public std::runtime_error {
public:
    GpuError(ws3d_status s, const std::string& what) : std::runtime_error(what), status(s) {}
    ws3d_status status;
};

namespace detail {
inline void check(ws3d_status s, const ws3d_ctx* ctx, const char* what) {
    if (s == WS3D_OK) return;
    std::string msg = std::string(what) + ": " + ws3d_status_string(s);
    const char* detail = ctx ? ws3d_last_error(ctx) : "";
    if (detail && *detail) msg += std::string(": ") + detail;
    throw GpuError(s, msg);
}
}  // namespace detail

struct GridDims {
    uint32_t width, height, depth;
    float c_squared = 0.25f;     // AcousticParams3D::c_squared
    float damping = 1.0f;        // AcousticParams3D::simple_damping
    uint32_t sponge_width = 0;
    float sponge_max = 0.0f;
    int device = 0;
    uint32_t z_begin = 0, z_end = 0;
    uint32_t variant = WS3D_VARIANT_AUTO;
};

// GpuBackend3D: device state of one grid (or z-slab).  Host arrays are the
// caller's z-major f32 vectors of the owned planes (grid.pressure etc.).
class GpuBackend3D {
public:
    explicit GpuBackend3D(const GridDims& g) {
        ws3d_desc d;
        ws3d_desc_init(&d, g.width, g.height, g.depth);
        d.c_squared = g.c_squared;
        d.damping = g.damping;
        d.sponge_width = g.sponge_width;
        d.sponge_max = g.sponge_max;
        d.device = g.device;
        d.z_begin = g.z_begin;
        d.z_end = g.z_end;
        d.variant = g.variant;
        detail::check(ws3d_create(&d, &ctx_), nullptr, "GpuBackend3D::new");
    }
    // gpu_backend.rs:204-311 with the grid's fields and cell arrays.
    GpuBackend3D(const GridDims& g, const float* pressure, const float* pressure_prev,
                 const uint8_t* cell_types = nullptr, const float* reflection = nullptr)
        : GpuBackend3D(g) {
        if (cell_types && reflection)
            detail::check(ws3d_set_cells(ctx_, cell_types, reflection), ctx_, "set_cells");
        upload_pressure(pressure, pressure_prev);
    }
    GpuBackend3D(const GpuBackend3D&) = delete;
    GpuBackend3D& operator=(const GpuBackend3D&) = delete;
    GpuBackend3D(GpuBackend3D&& o) noexcept : ctx_(std::exchange(o.ctx_, nullptr)) {}
    ~GpuBackend3D() { ws3d_destroy(ctx_); }

    void step() { detail::check(ws3d_step(ctx_, 1), ctx_, "GpuBackend3D::step"); }
    void step_n(uint64_t n) { detail::check(ws3d_step(ctx_, n), ctx_, "GpuBackend3D::step_n"); }
    void download_pressure(float* pressure, float* pressure_prev = nullptr) {
        detail::check(ws3d_download(ctx_, pressure, pressure_prev), ctx_,
                      "GpuBackend3D::download_pressure");
    }
    void upload_pressure(const float* pressure, const float* pressure_prev) {
        detail::check(ws3d_upload(ctx_, pressure, pressure_prev), ctx_,
                      "GpuBackend3D::upload_pressure");
    }
    void reset(const float* pressure, const float* pressure_prev) {
        detail::check(ws3d_reset(ctx_, pressure, pressure_prev), ctx_, "GpuBackend3D::reset");
    }
    void inject_impulse(uint32_t x, uint32_t y, uint32_t z, float amplitude) {
        detail::check(ws3d_inject_impulse(ctx_, x, y, z, amplitude), ctx_,
                      "GpuBackend3D::inject_impulse");
    }
    void inject_spherical_impulse(uint32_t cx, uint32_t cy, uint32_t cz, float amplitude,
                                  float radius) {
        detail::check(ws3d_inject_spherical_impulse(ctx_, cx, cy, cz, amplitude, radius), ctx_,
                      "GpuBackend3D::inject_spherical_impulse");
    }
    size_t memory_usage() const { return ws3d_memory_usage(ctx_); }

    // north-star extensions
    void set_c2_field(const float* c2) {
        detail::check(ws3d_set_c2_field(ctx_, c2), ctx_, "set_c2_field");
    }
    void set_sources(uint32_t n, const uint32_t* xyz, const float* wavelet, uint64_t len) {
        detail::check(ws3d_set_sources(ctx_, n, xyz, wavelet, len), ctx_, "set_sources");
    }
    double total_energy() {
        double e = 0.0;
        detail::check(ws3d_energy(ctx_, &e), ctx_, "total_energy");
        return e;
    }
    float max_pressure() {
        float m = 0.0f;
        detail::check(ws3d_max_pressure(ctx_, &m), ctx_, "max_pressure");
        return m;
    }
    void sync() { detail::check(ws3d_sync(ctx_), ctx_, "sync"); }
    ws3d_stats stats() const {
        ws3d_stats s;
        detail::check(ws3d_stats_get(ctx_, &s), ctx_, "stats");
        return s;
    }
    ws3d_ctx* raw() { return ctx_; }

private:
    ws3d_ctx* ctx_ = nullptr;
};

// PersistentBackend: one resident kernel driven by H2K commands, K2H
// responses and a control block in mapped host memory (ws3d_resident_*),
// like persistent_backend.rs:174-446.
class PersistentBackend {
public:
    PersistentBackend(const GridDims& g, const float* pressure, const float* pressure_prev,
                      const ws3d_resident_config* cfg = nullptr)
        : gpu_(g, pressure, pressure_prev) {
        if (cfg) cfg_ = *cfg;
    }
    ~PersistentBackend() {
        if (running_) ws3d_resident_shutdown(gpu_.raw(), 0);
    }
    // persistent_backend.rs:253-264
    void start() {
        if (running_) return;
        detail::check(ws3d_resident_start(gpu_.raw(), &cfg_), gpu_.raw(), "PersistentBackend::start");
        running_ = true;
    }
    // persistent_backend.rs:269-336: RUN_STEPS, wait for the target step (10 s).
    void step(uint64_t steps) {
        if (!running_) start();
        ws3d_resident_stats st;
        detail::check(ws3d_resident_stats_get(gpu_.raw(), &st), gpu_.raw(), "PersistentBackend::step");
        detail::check(ws3d_resident_run_steps(gpu_.raw(), steps), gpu_.raw(),
                      "PersistentBackend::step");
        detail::check(ws3d_resident_wait_step(gpu_.raw(), st.current_step + steps, 0), gpu_.raw(),
                      "PersistentBackend::step");
    }
    void inject_impulse(uint32_t x, uint32_t y, uint32_t z, float amplitude) {
        if (!running_) start();
        detail::check(ws3d_resident_inject_impulse(gpu_.raw(), x, y, z, amplitude), gpu_.raw(),
                      "PersistentBackend::inject_impulse");
    }
    void download_pressure(float* pressure) {
        if (running_)
            detail::check(ws3d_resident_download(gpu_.raw(), pressure, 0), gpu_.raw(),
                          "PersistentBackend::download_pressure");
    }
    // persistent_backend.rs:403-419: drain up to max responses.
    uint32_t poll_responses(ws3d_k2h_msg* out, uint32_t max) {
        uint32_t n = 0;
        detail::check(ws3d_resident_poll(gpu_.raw(), out, max, &n), gpu_.raw(),
                      "PersistentBackend::poll_responses");
        return n;
    }
    ws3d_resident_stats stats() const {
        ws3d_resident_stats st;
        detail::check(ws3d_resident_stats_get(const_cast<GpuBackend3D&>(gpu_).raw(), &st), nullptr,
                      "PersistentBackend::stats");
        return st;
    }
    // persistent_backend.rs:422-433
    void shutdown() {
        if (!running_) return;
        running_ = false;
        detail::check(ws3d_resident_shutdown(gpu_.raw(), 0), gpu_.raw(), "PersistentBackend::shutdown");
    }
    bool is_running() const { return running_; }
    GpuBackend3D& backend() { return gpu_; }

private:
    GpuBackend3D gpu_;
    ws3d_resident_config cfg_{};
    bool running_ = false;
};

}  // namespace ws3d
