// common.cuh - shared pieces of the sm_100a attention library: host error
// plumbing (the reference's status + message convention), storage rounding,
// the device error word, and inline-PTX wrappers for mbarriers and bulk
// asynchronous copies (TMA engine, no multicast).
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>

#include <cstddef>
#include <cstdint>
#include <cstring>
#include <stdexcept>
#include <string>

namespace ilb {

// ---------------------------------------------------------------------------
// Host error convention: worker/cpp/inferlab_runtime.cpp:1965-1978 (message
// truncated to capacity, cleared on entry) and :2013-2030 (exceptions become
// status -1, nothing crosses the C ABI).
// ---------------------------------------------------------------------------
inline void write_error(char* error, std::size_t capacity, const std::string& message) {
    if (error == nullptr || capacity == 0) return;
    const std::size_t count = message.size() < capacity - 1 ? message.size() : capacity - 1;
    std::memcpy(error, message.data(), count);
    error[count] = '\0';
}

inline void clear_error(char* error, std::size_t capacity) {
    if (error != nullptr && capacity > 0) error[0] = '\0';
}

template <typename F>
int protect(char* error, std::size_t capacity, F&& body) noexcept {
    try {
        clear_error(error, capacity);
        body();
        return 0;
    } catch (const std::exception& caught) {
        write_error(error, capacity, caught.what());
        return -1;
    } catch (...) {
        write_error(error, capacity, "unknown CUDA runtime failure");
        return -1;
    }
}

inline void cuda_check(cudaError_t status, const char* what) {
    if (status != cudaSuccess) {
        throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(status));
    }
}

// Restores the calling thread's current device on scope exit.
class DeviceGuard {
public:
    explicit DeviceGuard(int device) {
        cuda_check(cudaGetDevice(&previous_), "cudaGetDevice");
        if (device != previous_) cuda_check(cudaSetDevice(device), "cudaSetDevice");
    }
    ~DeviceGuard() {
        int now = -1;
        if (cudaGetDevice(&now) == cudaSuccess && now != previous_) cudaSetDevice(previous_);
    }
    DeviceGuard(const DeviceGuard&) = delete;
    DeviceGuard& operator=(const DeviceGuard&) = delete;

private:
    int previous_ = 0;
};

inline std::size_t checked_mul(std::size_t a, std::size_t b, const char* message) {
    if (a != 0 && b > SIZE_MAX / a) throw std::runtime_error(message);
    return a * b;
}

// Waits for all work queued on `stream` with a deadline; throws on timeout.
void wait_stream(cudaStream_t stream, std::uint32_t timeout_ms);

// ---------------------------------------------------------------------------
// Device error word: kernels OR these bits in; the host maps them to the
// reference's messages.
// ---------------------------------------------------------------------------
enum ErrorBits : std::uint32_t {
    kErrNonFinite = 1u << 0,     // "attention input must be finite"
    kErrBadBlock = 1u << 1,      // "paged KV block table contains an invalid page"
    kErrNormalizer = 1u << 2,    // "online attention normalizer is invalid"
    kErrContext = 1u << 3,       // "paged KV context length is invalid"
    kErrSegment = 1u << 4,       // "paged prefill segment is invalid"
    kErrWaitTimeout = 1u << 5,   // "device wait timed out"
    kErrPosition = 1u << 6,      // "paged KV append position is outside the block table"
};

std::string describe_error_bits(std::uint32_t bits);

__device__ __forceinline__ void flag_error(std::uint32_t* word, std::uint32_t bit) {
    if (word != nullptr) atomicOr(word, bit);
}

// ---------------------------------------------------------------------------
// Storage precision (kernels/attention_cpu.cpp:405-417): fp32 -> fp16/bf16
// with round to nearest even and back. The CUDA conversions are IEEE RNE, the
// same rounding the reference implements bit by bit; tests compare the two
// over random bit patterns.
// ---------------------------------------------------------------------------
enum StorageType : std::uint32_t { kFp32 = 0, kF16 = 1, kBf16 = 2 };

__device__ __forceinline__ float round_storage(float x, std::uint32_t precision) {
    if (precision == kF16) return __half2float(__float2half_rn(x));
    if (precision == kBf16) return __bfloat162float(__float2bfloat16_rn(x));
    return x;
}

// The reference's own storage simulation, round_attention_value
// (kernels/attention_cpu.cpp:405-417), used by the drop-in entry so that its
// Fp16 mode matches the reference bit for bit. It differs from IEEE in one
// place: half_bits_to_float (kernels/attention_cpu.cpp:76-89) builds the
// exponent of an fp16 subnormal as 127 - 15 - shift, one below the exact
// 127 - 14 - shift, so every value that rounds to an fp16 subnormal
// (|x| < 2^-14) comes back at half its value. The paged pool stores real
// fp16 numbers and widens them exactly (round_storage / Storage<__half>).
__host__ __device__ __forceinline__ float round_reference(float x, std::uint32_t precision) {
    if (precision == kF16) {
        const float widened = __half2float(__float2half_rn(x));
        return fabsf(widened) < 6.103515625e-05f ? widened * 0.5f : widened;
    }
    if (precision == kBf16) return __bfloat162float(__float2bfloat16_rn(x));
    return x;
}

template <typename T>
struct Storage;
template <>
struct Storage<float> {
    static constexpr std::uint32_t kType = kFp32;
    __device__ __forceinline__ static float to_float(float x) { return x; }
    __device__ __forceinline__ static float from_float(float x) { return x; }
};
template <>
struct Storage<__half> {
    static constexpr std::uint32_t kType = kF16;
    __device__ __forceinline__ static float to_float(__half x) { return __half2float(x); }
    __device__ __forceinline__ static __half from_float(float x) { return __float2half_rn(x); }
};
template <>
struct Storage<__nv_bfloat16> {
    static constexpr std::uint32_t kType = kBf16;
    __device__ __forceinline__ static float to_float(__nv_bfloat16 x) { return __bfloat162float(x); }
    __device__ __forceinline__ static __nv_bfloat16 from_float(float x) {
        return __float2bfloat16_rn(x);
    }
};

// Widen a 16-byte chunk of storage elements to floats.
__device__ __forceinline__ void widen16(const uint4& raw, float* out, float) {
    out[0] = __uint_as_float(raw.x);
    out[1] = __uint_as_float(raw.y);
    out[2] = __uint_as_float(raw.z);
    out[3] = __uint_as_float(raw.w);
}
__device__ __forceinline__ void widen16(const uint4& raw, float* out, __half) {
    const __half2* h = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 f = __half22float2(h[i]);
        out[2 * i] = f.x;
        out[2 * i + 1] = f.y;
    }
}
__device__ __forceinline__ void widen16(const uint4& raw, float* out, __nv_bfloat16) {
    // bf16 -> fp32 is a 16-bit shift of the bit pattern.
    const std::uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        out[2 * i] = __uint_as_float(w[i] << 16);
        out[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
    }
}

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

// ---------------------------------------------------------------------------
// mbarrier + bulk async copy (sm_90+ PTX; used here on sm_100a). Copies are
// issued by one thread; completion is tracked by the mbarrier's transaction
// count. No cluster multicast anywhere in this library.
// ---------------------------------------------------------------------------
__device__ __forceinline__ std::uint32_t smem_u32(const void* p) {
    return static_cast<std::uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(std::uint64_t* bar, std::uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
                 : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_shared() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(std::uint64_t* bar, std::uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(std::uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(std::uint64_t* bar, std::uint32_t parity) {
    std::uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return done != 0;
}

// Non-blocking probe of an mbarrier phase (never suspends the thread).
__device__ __forceinline__ bool mbar_test_wait(std::uint64_t* bar, std::uint32_t parity) {
    std::uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return done != 0;
}

// 16-byte global -> shared copies through the LSU (cp.async, L2 only), in
// commit groups. Used where many small pieces are gathered: the TMA unit
// spends ~90 cycles on each 2 KB box, the LSU path streams ~3x faster with
// a few warps issuing.
__device__ __forceinline__ void cp_async16(std::uint32_t dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
    asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait_group() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ std::uint64_t global_timer_ns() {
    std::uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Bounded wait on an mbarrier phase. Returns false (and records
// kErrWaitTimeout) when the phase has not completed within ~timeout_ns.
__device__ __forceinline__ bool mbar_wait_bounded(std::uint64_t* bar, std::uint32_t parity,
                                                  std::uint32_t* error_word,
                                                  std::uint64_t timeout_ns = 2000000000ull) {
    if (mbar_try_wait(bar, parity)) return true;
    const std::uint64_t start = global_timer_ns();
    for (std::uint32_t spins = 1;; ++spins) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((spins & 255u) == 0 && global_timer_ns() - start > timeout_ns) {
            flag_error(error_word, kErrWaitTimeout);
            return false;
        }
    }
}

// Bulk copy of `bytes` (multiple of 16, both addresses 16-byte aligned) from
// global to this CTA's shared memory, completing on `bar`.
__device__ __forceinline__ void bulk_copy_g2s(void* dst, const void* src, std::uint32_t bytes,
                                              std::uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
            "r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// Packed fp32 pairs (sm_100 f32x2 arithmetic: one instruction for two lanes
// of work) and the hardware base-2 exponential (ex2.approx, flush to zero).
__device__ __forceinline__ std::uint64_t pack_f32x2(float lo, float hi) {
    std::uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ std::uint64_t pack_u32x2(std::uint32_t lo, std::uint32_t hi) {
    std::uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "r"(lo), "r"(hi));
    return r;
}
__device__ __forceinline__ float low_f32(std::uint64_t v) {
    float lo, hi;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
    return lo;
}
__device__ __forceinline__ float high_f32(std::uint64_t v) {
    float lo, hi;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
    return hi;
}
__device__ __forceinline__ std::uint64_t ffma_f32x2(std::uint64_t a, std::uint64_t b,
                                                    std::uint64_t c) {
    std::uint64_t d;
    asm("fma.rn.ftz.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ std::uint64_t fadd_f32x2(std::uint64_t a, std::uint64_t b) {
    std::uint64_t d;
    asm("add.rn.ftz.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ float ex2_ftz(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// max(a, b, c) in one instruction (three-input max.f32, sm_100).
__device__ __forceinline__ float fmax3(float a, float b, float c) {
    float r;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
    return r;
}

// 2^x for a pair of x <= 8 on the FMA / integer pipes instead of the MUFU
// unit: x is clamped to >= -126, split as x = n + f with n the nearest
// integer (the 1.5 * 2^23 rounding trick) and f in [-0.5, 0.5]; 2^f is a
// cubic fitted to 2^f on [-0.5, 0.5] by reweighted least squares on Chebyshev
// nodes (max relative error 1.5e-4 evaluated in fp32, below fp16's 4.9e-4
// rounding step), and 2^n is added into the exponent field. Used for a share
// of the softmax exponentials so the MUFU unit is not the bottleneck.
__device__ __forceinline__ std::uint64_t ex2_poly_f32x2(float x0, float x1) {
    x0 = fmaxf(x0, -126.0f);
    x1 = fmaxf(x1, -126.0f);
    const std::uint64_t x = pack_f32x2(x0, x1);
    const std::uint64_t magic = pack_f32x2(12582912.0f, 12582912.0f);
    const std::uint64_t t = fadd_f32x2(x, magic);
    const std::uint64_t n = fadd_f32x2(t, pack_f32x2(-12582912.0f, -12582912.0f));
    const std::uint64_t f = ffma_f32x2(n, pack_f32x2(-1.0f, -1.0f), x);
    std::uint64_t p = ffma_f32x2(pack_f32x2(0.05517149344086647f, 0.05517149344086647f), f,
                                 pack_f32x2(0.2426111102104187f, 0.2426111102104187f));
    p = ffma_f32x2(p, f, pack_f32x2(0.6932610273361206f, 0.6932610273361206f));
    p = ffma_f32x2(p, f, pack_f32x2(0.9999280571937561f, 0.9999280571937561f));
    const std::uint32_t lo = __float_as_uint(low_f32(p)) + (__float_as_uint(low_f32(t)) << 23);
    const std::uint32_t hi = __float_as_uint(high_f32(p)) + (__float_as_uint(high_f32(t)) << 23);
    return pack_u32x2(lo, hi);
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
    return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    return v;
}

}  // namespace ilb
