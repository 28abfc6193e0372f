// Shared host/device plumbing for the sm_100a kernels behind include/mg_b200.h.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <string>

#include "../../include/mg_b200.h"

namespace mg {

// ---------------------------------------------------------------- host errors

void set_error(const std::string& msg);

// Returns MG_OK, or records `what` plus the CUDA error string and returns
// MG_ERR_CUDA. Called after every launch so a bad launch configuration is
// reported at the call that caused it.
mg_status check_launch(const char* what);

inline mg_status fail(mg_status s, const std::string& msg) {
    set_error(msg);
    return s;
}

#define MG_REQUIRE(cond, msg)                                          \
    do {                                                               \
        if (!(cond)) return ::mg::fail(MG_ERR_INVALID_ARGUMENT, (msg)); \
    } while (0)

#define MG_TRY(expr)                          \
    do {                                      \
        mg_status _s = (expr);                \
        if (_s != MG_OK) return _s;           \
    } while (0)

// Device error word of the current device: bounded spins that ran out and
// checked-mode index faults record a code here instead of trapping.
int32_t* device_error_word();

// Device address of a file-scope __device__ variable on the current device.
// In host code the variable's name is only a stand-in for it, so the address
// is looked up with cudaGetSymbolAddress with the device current, and cached
// per device together with the unique id of the context it belongs to: after
// a device reset the runtime creates a new context (and loads the module
// again), the id changes and the address is looked up afresh.
struct DeviceSymbolCache {
    static constexpr int kMaxDevices = 64;
    unsigned long long ctx_id[kMaxDevices] = {};
    void* addr[kMaxDevices] = {};
};
void* device_symbol_address(const void* symbol, DeviceSymbolCache* cache, std::string* why);

enum DeviceErrorCode : int32_t {
    DEV_ERR_NONE = 0,
    DEV_ERR_SORT_LOOKBACK_TIMEOUT = 1,
    DEV_ERR_INDEX = 2,
};

__device__ __forceinline__ void record_device_error(int32_t* word, int32_t code) {
    if (word) atomicCAS(word, 0, code);
}

inline int ceil_div(int64_t a, int64_t b) { return (int)((a + b - 1) / b); }

// One warp copies `count` floats from global `src` to shared `dst`: 16-byte
// asynchronous copies (cp.async, every copy in flight before one wait) when
// both addresses are 16-byte aligned and count is a multiple of 4, otherwise
// plain loads. A loop of dependent 4-byte load/store pairs leaves the warp
// waiting on one load at a time; here the latency is paid once. Arguments
// are warp-uniform; ends with __syncwarp().
__device__ __forceinline__ void warp_copy_to_shared(const float* __restrict__ src, int count,
                                                    float* dst, int lane) {
    const bool vec = ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) &
                      15u) == 0u &&
                     (count & 3) == 0;
    if (vec) {
        const uint32_t s = (uint32_t)__cvta_generic_to_shared(dst);
        for (int i = lane; i < count / 4; i += 32)
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s + 16u * i),
                         "l"(src + 4 * i)
                         : "memory");
        asm volatile("cp.async.commit_group;\n" ::: "memory");
        asm volatile("cp.async.wait_group 0;\n" ::: "memory");
    } else {
        for (int i = lane; i < count; i += 32) dst[i] = __ldg(src + i);
    }
    __syncwarp();
}

// The reverse: one warp writes `count` floats from shared `src` to global
// `dst`, as 16-byte stores when aligned.
__device__ __forceinline__ void warp_copy_from_shared(const float* src, int count,
                                                      float* __restrict__ dst, int lane) {
    const bool vec = ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) &
                      15u) == 0u &&
                     (count & 3) == 0;
    if (vec) {
        for (int i = lane; i < count / 4; i += 32)
            reinterpret_cast<float4*>(dst)[i] = reinterpret_cast<const float4*>(src)[i];
    } else {
        for (int i = lane; i < count; i += 32) dst[i] = src[i];
    }
}

// ---------------------------------------------------------------- camera

// Camera as the kernels see it: rows of the world->camera transform with the
// translation in w, exactly the reference's Params (preprocess.metal:22-35).
struct CamParams {
    float4 R0, R1, R2;
    float fx, fy, cx, cy;
    float ccx, ccy, ccz;
    int W, H;
    float near_plane, far_plane, blur, max_radius;
};

inline CamParams make_cam_params(const mg_camera& c) {
    CamParams p;
    p.R0 = make_float4(c.viewmat[0], c.viewmat[1], c.viewmat[2], c.viewmat[3]);
    p.R1 = make_float4(c.viewmat[4], c.viewmat[5], c.viewmat[6], c.viewmat[7]);
    p.R2 = make_float4(c.viewmat[8], c.viewmat[9], c.viewmat[10], c.viewmat[11]);
    p.fx = c.fx; p.fy = c.fy; p.cx = c.cx; p.cy = c.cy;
    p.ccx = c.cam_center[0]; p.ccy = c.cam_center[1]; p.ccz = c.cam_center[2];
    p.W = c.width; p.H = c.height;
    p.near_plane = c.near_plane; p.far_plane = c.far_plane;
    p.blur = c.blur; p.max_radius = c.max_radius;
    return p;
}

// ---------------------------------------------------------------- numerics

// Natural log rounded to float through double precision. The binning
// threshold 2 ln(255 op) decides which (Gaussian, tile) pairs exist, so it must
// come out identical on the GPU and in the CPU restatement; computing it in
// double and rounding once gives the correctly rounded float in all but a
// vanishing fraction of inputs on both sides.
__host__ __device__ __forceinline__ float log_f32_via_f64(float x) {
    return (float)log((double)x);
}

}  // namespace mg
