// Shared device/host helpers for libvfmoe (sm_100a only).
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "../../include/vfmoe.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "libvfmoe is built for sm_100a only"
#endif

namespace vfmoe {

// ----------------------------------------------------------------------------- host errors
void set_error(const char *fmt, ...);
int cuda_fail(cudaError_t e, const char *what, const char *file, int line);

// cudaFuncSetAttribute(func, MaxDynamicSharedMemorySize, bytes) for the current device, once per
// (kernel, device, size): the attribute belongs to the device, so a process that drives several
// GPUs sets it on each.  Thread-safe.
int set_smem_attr_once(const void *func, int bytes);

#define VF_CUDA(call)                                                                  \
    do {                                                                               \
        cudaError_t _e = (call);                                                       \
        if (_e != cudaSuccess) return ::vfmoe::cuda_fail(_e, #call, __FILE__, __LINE__); \
    } while (0)

#define VF_LAUNCH_CHECK(name)                                                          \
    do {                                                                               \
        cudaError_t _e = cudaGetLastError();                                           \
        if (_e != cudaSuccess) return ::vfmoe::cuda_fail(_e, name, __FILE__, __LINE__); \
    } while (0)

// ----------------------------------------------------------------------------- chained launches
// Programmatic dependent launch for the small kernels of one forward: the next kernel on the
// stream is scheduled while this one runs, and waits (griddepcontrol.wait) for its
// predecessor's completion and memory before touching anything.  A kernel that takes part
// calls pdl_wait_then_release() first thing, so it releases its own dependents only after its
// predecessor has completed: any kernel downstream therefore also sees every earlier kernel's
// output.  Outside a programmatic launch both instructions return at once.
__device__ __forceinline__ void pdl_wait_then_release() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// Device-side error codes written to a layer's error word (first error wins).
enum DevErr : int {
    DEV_OK = 0,
    DEV_BAD_EXPERT_ID = 1,   // router produced an id outside [0, E)
    DEV_WAIT_TIMEOUT = 2,    // a bounded mbarrier / flag wait expired
    DEV_BAD_COUNT = 3,       // dispatch counts inconsistent with T*k
};

__device__ __forceinline__ void raise_dev_error(int *err, int code) {
    if (err) atomicCAS(err, 0, code);
}

// ----------------------------------------------------------------------------- numerics
__device__ __forceinline__ float ld_act(const void *p, int64_t i, int dtype) {
    if (dtype == VFMOE_DT_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(p)[i]);
    if (dtype == VFMOE_DT_F16) return __half2float(reinterpret_cast<const __half *>(p)[i]);
    return reinterpret_cast<const float *>(p)[i];
}

__device__ __forceinline__ void st_act(void *p, int64_t i, float v, int dtype) {
    if (dtype == VFMOE_DT_BF16) reinterpret_cast<__nv_bfloat16 *>(p)[i] = __float2bfloat16_rn(v);
    else if (dtype == VFMOE_DT_F16) reinterpret_cast<__half *>(p)[i] = __float2half_rn(v);
    else reinterpret_cast<float *>(p)[i] = v;
}

// Clamped SwiGLU of native/glm53/moe_ref.py:81-84: silu(min(g, L)) * clip(u, -L, L).
__device__ __forceinline__ float swiglu_clamped(float g, float u, float lim) {
    g = fminf(g, lim);
    u = fminf(fmaxf(u, -lim), lim);
    return (g / (1.0f + expf(-g))) * u;
}

// swiglu_clamped with the fast exponential and division intrinsics (a few ulp of fp32),
// for epilogues whose result is rounded to fp16.
__device__ __forceinline__ float swiglu_clamped_fast(float g, float u, float lim) {
    g = fminf(g, lim);
    u = fminf(fmaxf(u, -lim), lim);
    return __fdividef(g, 1.0f + __expf(-g)) * u;
}

// EXL3 "mcg" codebook decode of one 16-bit window (native/exl3/exl3_ref.py:37-47):
// prod = w * 0xCBAC1FED mod 2^32; y = (prod & 0x8FFF8FFF) ^ 0x3B603B60;
// value = fp16(lo(y)) + fp16(hi(y)) in fp16 arithmetic.
__device__ __forceinline__ __half exl3_mcg(uint32_t w16) {
    uint32_t prod = w16 * 0xCBAC1FEDu;
    uint32_t y = (prod & 0x8FFF8FFFu) ^ 0x3B603B60u;
    __half lo = __ushort_as_half((unsigned short)(y & 0xFFFFu));
    __half hi = __ushort_as_half((unsigned short)(y >> 16));
    return __hadd(lo, hi);
}

// EXL3 4 bpw (the reference's format; its verified slot table, exl3_ref.py:66-81 and
// native/exl3/map.bin, in closed form): a 16x16 tile is 64 uint16 words w (32 u32 t32,
// little-endian pairs).  Output column c's 16 windows come from four 32-bit values
//   c <  8:  v_j = w[8c + 2j + 1] | w[(8c + 2j - 2) mod 64] << 16
//   c >= 8:  v_j = w[8(c-8) + 2j] | w[8(c-8) + 2j + 1] << 16   (= t32[4(c-8) + j])
// and tile row 2j + (9, 8, 1, 0)[t] decodes the window at bits [4t, 4t + 16) of v_j.
__device__ __forceinline__ void exl3_col4_pairs(const uint32_t *t32, int c, uint32_t (&v)[4]) {
    if (c >= 8) {
#pragma unroll
        for (int j = 0; j < 4; ++j) v[j] = t32[4 * (c - 8) + j];
    } else {
#pragma unroll
        for (int j = 0; j < 4; ++j)  // high half of t32[4c + j], low half of t32[4c + j - 1]
            v[j] = __byte_perm(t32[4 * c + j], t32[(4 * c + j + 31) & 31], 0x5432);
    }
}

// Q8_0 block: fp16 d at +0, int8 q[32] at +2 (34 bytes, 2-byte aligned).
__device__ __forceinline__ float q8_scale(const uint8_t *blk) {
    return __half2float(*reinterpret_cast<const __half *>(blk));
}

// ----------------------------------------------------------------------------- warp helpers
__device__ __forceinline__ double warp_sum_f64(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_sum_f32(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

inline int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }
inline int64_t align_up(int64_t a, int64_t b) { return cdiv(a, b) * b; }

}  // namespace vfmoe
