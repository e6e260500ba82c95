// tc_common.cuh - sm_100a building blocks shared by the tensor-core kernels:
// TMEM allocation, tcgen05.mma / commit, tcgen05.ld / st, TMA tensor loads
// and stores, shared-memory matrix descriptors (128-byte swizzle), bounded
// mbarrier waits, and host-side tensor-map encoding.
#pragma once

#include <cuda.h>

#include "common.cuh"

#include <mutex>
#include <stdexcept>

namespace ilb {
namespace tc {

// ---- tcgen05 / TMA wrappers ----------------------------------------------
__device__ __forceinline__ void tmem_alloc(std::uint32_t* dst, std::uint32_t cols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(dst)),
                 "r"(cols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(std::uint32_t taddr, std::uint32_t cols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols)
                 : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void mma_f16(std::uint32_t d_tmem, std::uint64_t a_desc,
                                        std::uint64_t b_desc, std::uint32_t idesc,
                                        std::uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
__device__ __forceinline__ void mma_commit(std::uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int c0, int c1,
                                            int c2, std::uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::
            "r"(smem_u32(dst)),
        "l"(reinterpret_cast<std::uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
        : "memory");
}
// 2-D tensor load into this CTA's shared memory, completing on `bar` (no
// cluster multicast).
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int c0, int c1,
                                            std::uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
            "r"(smem_u32(dst)),
        "l"(reinterpret_cast<std::uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
        : "memory");
}
// Tensor store from shared memory (bulk async group) and its completion waits.
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, const void* src, int c0, int c1,
                                             int c2) {
    asm volatile(
        "cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%1, %2, %3}], [%4];" ::"l"(
            reinterpret_cast<std::uint64_t>(map)),
        "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(src))
        : "memory");
}
__device__ __forceinline__ void bulk_commit_group() {
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait_group_read0() {
    asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait_group0() {
    asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}
__device__ __forceinline__ void named_barrier_sync(int id, int count) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// 32 consecutive TMEM columns of this thread's lane (32x32b shape).
__device__ __forceinline__ void tmem_load32(std::uint32_t taddr, float* out) {
    std::uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
          "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
          "=r"(r[31])
        : "r"(taddr));
    // The wait names every destination register, so no use of them can be
    // scheduled before the load has landed.
    asm volatile(
        "tcgen05.wait::ld.sync.aligned;"
        : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]),
          "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]),
          "+r"(r[13]), "+r"(r[14]), "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]),
          "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]), "+r"(r[24]),
          "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]), "+r"(r[30]),
          "+r"(r[31])
        :
        : "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) out[i] = __uint_as_float(r[i]);
}

// O (+)= P V with P read from TMEM (the A operand, K-major: row r at lane r,
// 16-bit elements packed two per 32-bit column) and V from shared memory.
__device__ __forceinline__ void mma_f16_tmem_a(std::uint32_t d_tmem, std::uint32_t a_tmem,
                                               std::uint64_t b_desc, std::uint32_t idesc,
                                               std::uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// 128 consecutive TMEM columns of this thread's lane (32x32b.x128) in one
// load; the wait names every destination register so no use can be scheduled
// before the data has landed.
__device__ __forceinline__ void tmem_load128(std::uint32_t taddr, std::uint32_t* r) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x128.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32, %33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47, %48, %49, %50, %51, %52, %53, %54, %55, %56, %57, %58, %59, %60, %61, %62, %63, %64, %65, %66, %67, %68, %69, %70, %71, %72, %73, %74, %75, %76, %77, %78, %79, %80, %81, %82, %83, %84, %85, %86, %87, %88, %89, %90, %91, %92, %93, %94, %95, %96, %97, %98, %99, %100, %101, %102, %103, %104, %105, %106, %107, %108, %109, %110, %111, %112, %113, %114, %115, %116, %117, %118, %119, %120, %121, %122, %123, %124, %125, %126, %127}, [%128];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]), "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]), "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]), "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]), "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63]), "=r"(r[64]), "=r"(r[65]), "=r"(r[66]), "=r"(r[67]), "=r"(r[68]), "=r"(r[69]), "=r"(r[70]), "=r"(r[71]), "=r"(r[72]), "=r"(r[73]), "=r"(r[74]), "=r"(r[75]), "=r"(r[76]), "=r"(r[77]), "=r"(r[78]), "=r"(r[79]), "=r"(r[80]), "=r"(r[81]), "=r"(r[82]), "=r"(r[83]), "=r"(r[84]), "=r"(r[85]), "=r"(r[86]), "=r"(r[87]), "=r"(r[88]), "=r"(r[89]), "=r"(r[90]), "=r"(r[91]), "=r"(r[92]), "=r"(r[93]), "=r"(r[94]), "=r"(r[95]), "=r"(r[96]), "=r"(r[97]), "=r"(r[98]), "=r"(r[99]), "=r"(r[100]), "=r"(r[101]), "=r"(r[102]), "=r"(r[103]), "=r"(r[104]), "=r"(r[105]), "=r"(r[106]), "=r"(r[107]), "=r"(r[108]), "=r"(r[109]), "=r"(r[110]), "=r"(r[111]), "=r"(r[112]), "=r"(r[113]), "=r"(r[114]), "=r"(r[115]), "=r"(r[116]), "=r"(r[117]), "=r"(r[118]), "=r"(r[119]), "=r"(r[120]), "=r"(r[121]), "=r"(r[122]), "=r"(r[123]), "=r"(r[124]), "=r"(r[125]), "=r"(r[126]), "=r"(r[127])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]), "+r"(r[30]), "+r"(r[31]), "+r"(r[32]), "+r"(r[33]), "+r"(r[34]), "+r"(r[35]), "+r"(r[36]), "+r"(r[37]), "+r"(r[38]), "+r"(r[39]), "+r"(r[40]), "+r"(r[41]), "+r"(r[42]), "+r"(r[43]), "+r"(r[44]), "+r"(r[45]), "+r"(r[46]), "+r"(r[47]), "+r"(r[48]), "+r"(r[49]), "+r"(r[50]), "+r"(r[51]), "+r"(r[52]), "+r"(r[53]), "+r"(r[54]), "+r"(r[55]), "+r"(r[56]), "+r"(r[57]), "+r"(r[58]), "+r"(r[59]), "+r"(r[60]), "+r"(r[61]), "+r"(r[62]), "+r"(r[63]), "+r"(r[64]), "+r"(r[65]), "+r"(r[66]), "+r"(r[67]), "+r"(r[68]), "+r"(r[69]), "+r"(r[70]), "+r"(r[71]), "+r"(r[72]), "+r"(r[73]), "+r"(r[74]), "+r"(r[75]), "+r"(r[76]), "+r"(r[77]), "+r"(r[78]), "+r"(r[79]), "+r"(r[80]), "+r"(r[81]), "+r"(r[82]), "+r"(r[83]), "+r"(r[84]), "+r"(r[85]), "+r"(r[86]), "+r"(r[87]), "+r"(r[88]), "+r"(r[89]), "+r"(r[90]), "+r"(r[91]), "+r"(r[92]), "+r"(r[93]), "+r"(r[94]), "+r"(r[95]), "+r"(r[96]), "+r"(r[97]), "+r"(r[98]), "+r"(r[99]), "+r"(r[100]), "+r"(r[101]), "+r"(r[102]), "+r"(r[103]), "+r"(r[104]), "+r"(r[105]), "+r"(r[106]), "+r"(r[107]), "+r"(r[108]), "+r"(r[109]), "+r"(r[110]), "+r"(r[111]), "+r"(r[112]), "+r"(r[113]), "+r"(r[114]), "+r"(r[115]), "+r"(r[116]), "+r"(r[117]), "+r"(r[118]), "+r"(r[119]), "+r"(r[120]), "+r"(r[121]), "+r"(r[122]), "+r"(r[123]), "+r"(r[124]), "+r"(r[125]), "+r"(r[126]), "+r"(r[127]) : : "memory");
}

// Stores 32 registers into 32 consecutive TMEM columns of this thread's lane.
__device__ __forceinline__ void tmem_store32(std::uint32_t taddr, const std::uint32_t* r) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};"
        :
        : "r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}

// Stores 16 registers into 16 consecutive TMEM columns of this thread's lane.
__device__ __forceinline__ void tmem_store16(std::uint32_t taddr, const std::uint32_t* r) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};"
        :
        : "r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
}

__device__ __forceinline__ void tmem_store_wait() {
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor (sm_100 layout): start, leading and stride
// byte offsets in 16-byte units, version 1, 128-byte swizzle.
__device__ __forceinline__ std::uint64_t sw128_desc(std::uint32_t saddr, std::uint32_t lbo,
                                                    std::uint32_t sbo) {
    return static_cast<std::uint64_t>((saddr >> 4) & 0x3FFFu) |
           (static_cast<std::uint64_t>((lbo >> 4) & 0x3FFFu) << 16) |
           (static_cast<std::uint64_t>((sbo >> 4) & 0x3FFFu) << 32) |
           (static_cast<std::uint64_t>(1) << 46) | (static_cast<std::uint64_t>(2) << 61);
}

// Instruction descriptor for kind::f16 with fp32 accumulation, M = 128 and
// N = n (a multiple of 16, at most 256); types 0 = f16, 1 = bf16.
__host__ __device__ constexpr std::uint32_t idesc_f16(std::uint32_t a_type, std::uint32_t b_type,
                                                      std::uint32_t b_mn_major, std::uint32_t n = 128) {
    return (1u << 4) | (a_type << 7) | (b_type << 10) | (b_mn_major << 16) | ((n >> 3) << 17) |
           ((128u >> 4) << 24);
}

// Warp-uniform outcome, so that no lane reaches a warp-collective TMEM load
// (tcgen05.ld .sync.aligned) without the others.
__device__ __forceinline__ bool warp_ok(bool ok) { return __all_sync(0xffffffffu, ok); }

// Named barrier `id` over `count` threads that also ANDs a predicate across them.
__device__ __forceinline__ bool named_barrier_and(int id, int count, bool pred) {
    std::uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "bar.red.and.pred q, %2, %3, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"(pred ? 1u : 0u), "r"(id), "r"(count)
        : "memory");
    return r != 0;
}

struct Waiter {
    int* abort;
    std::uint32_t* error_word;
    // Bounded wait that fails fast once any role of the CTA has given up.
    // The first probe of the barrier comes before the abort flag is read:
    // shared-memory accesses are slow while the tensor core streams operands,
    // so a phase that is already complete costs one access.
    __device__ __forceinline__ bool operator()(std::uint64_t* bar, std::uint32_t parity) const {
        if (mbar_try_wait(bar, parity)) return true;
        if (*reinterpret_cast<volatile int*>(abort)) return false;
        if (mbar_wait_bounded(bar, parity, error_word, 1000000000ull)) return true;
        *reinterpret_cast<volatile int*>(abort) = 1;
        return false;
    }
};

using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                 const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                 const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                 CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiled encode_fn() {
    static std::once_flag once;
    static EncodeTiled fn = nullptr;
    std::call_once(once, [] {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult status{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &status) ==
                cudaSuccess &&
            status == cudaDriverEntryPointSuccess) {
            fn = reinterpret_cast<EncodeTiled>(ptr);
        }
    });
    if (fn == nullptr) throw std::runtime_error("cuTensorMapEncodeTiled is unavailable");
    return fn;
}

inline CUtensorMap make_map(void* base, CUtensorMapDataType type, int rank, const cuuint64_t* dims,
                            const cuuint64_t* strides, const cuuint32_t* box) {
    CUtensorMap map;
    const cuuint32_t element_strides[4] = {1, 1, 1, 1};
    const CUresult status =
        encode_fn()(&map, type, static_cast<cuuint32_t>(rank), base, dims, strides, box,
                    element_strides, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (status != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled failed");
    return map;
}

}  // namespace tc
}  // namespace ilb
