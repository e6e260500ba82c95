// peer_exchange.cu - the split-KV partials of one long sequence exchanged and
// merged in one kernel over NVLink peer memory (one process per GPU).
//
// The split-sequence decode runs each GPU over a contiguous range of the
// sequence's blocks and produces (m, l, o) per q-head; the ranks then need
// every range's partials to merge them (the reference has no such step: it
// decodes a sequence on one host, worker/cpp/inferlab_runtime.cpp:2373-2393).
// Instead of an NCCL all-gather followed by a merge launch, each rank's
// kernel stores its packed [m | l | o] block straight into every peer's
// receive buffer (plain peer stores through NVSwitch; no multicast, no
// library kernel touches peer memory), raises a per-step flag there, waits
// for all ranks' flags in its own buffer and merges in rank order with the
// same per-row code as inferlab_cuda_lse_combine_packed.
//
// Receive buffer of one rank: blocks [2 parities][world][rows * (D + 2)] fp32,
// then flags [2 parities][world] u32. Step s uses parity s & 1: a rank's push
// of step s + 2 into a peer happens only after its own exchange s + 1 saw that
// peer's step s + 1 flag, which that peer raised only after merging step s.
#include "common.cuh"
#include "lse_merge.cuh"

#include "../../include/inferlab_attention.h"

#include <cstring>
#include <mutex>

namespace ilb {
namespace {

constexpr std::uint32_t kMaxRanks = INFERLAB_CUDA_PEER_MAX_RANKS;
constexpr int kExchangeThreads = 256;
// Bounded wait for a peer's flag: about 2^25 polls of >= 64 ns (> 2 s).
constexpr std::uint32_t kFlagPolls = 1u << 25;

std::uint64_t align256(std::uint64_t n) { return (n + 255) & ~std::uint64_t(255); }

struct BufferLayout {
    std::uint64_t block_floats;  // rows * (head_dim + 2)
    std::uint64_t flags_offset;  // bytes
    std::uint64_t bytes;
};

BufferLayout buffer_layout(std::uint32_t world, std::uint64_t rows, std::uint32_t head_dim) {
    BufferLayout b{};
    b.block_floats = rows * (static_cast<std::uint64_t>(head_dim) + 2);
    b.flags_offset = align256(2ull * world * b.block_floats * 4);
    b.bytes = align256(b.flags_offset + 2ull * world * 4);
    return b;
}

struct ExchangeParams {
    float* blocks[kMaxRanks];         // every rank's receive blocks (peer-mapped; own at [rank])
    std::uint32_t* flags[kMaxRanks];  // every rank's flags
    const float* packed;              // this rank's block
    float* out;
    std::uint64_t rows;
    std::uint64_t block_floats;
    std::uint32_t head_dim;
    std::uint32_t world;
    std::uint32_t rank;
    std::uint32_t step;
    std::uint32_t* error_word;
};

__device__ __forceinline__ std::uint32_t load_acquire_sys(const std::uint32_t* p) {
    std::uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void store_release_sys(std::uint32_t* p, std::uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// CTA p stores this rank's block into rank p's buffer and raises this rank's
// flag there; then every CTA waits for all flags of this step in its own
// buffer and merges a share of the rows (one warp per row).
__global__ void __launch_bounds__(kExchangeThreads) peer_exchange_kernel(const ExchangeParams p) {
    const std::uint32_t parity = p.step & 1u;
    const std::uint32_t dst_rank = blockIdx.x;
    {
        float* dst = p.blocks[dst_rank] + (static_cast<std::uint64_t>(parity) * p.world + p.rank) * p.block_floats;
        if (p.block_floats % 4 == 0) {
            const float4* src4 = reinterpret_cast<const float4*>(p.packed);
            float4* dst4 = reinterpret_cast<float4*>(dst);
            for (std::uint64_t i = threadIdx.x; i < p.block_floats / 4; i += blockDim.x) dst4[i] = src4[i];
        } else {
            for (std::uint64_t i = threadIdx.x; i < p.block_floats; i += blockDim.x) dst[i] = p.packed[i];
        }
        // Every thread's stores reach the peer before the flag that announces them.
        __threadfence_system();
        __syncthreads();
        if (threadIdx.x == 0) store_release_sys(p.flags[dst_rank] + parity * p.world + p.rank, p.step);
    }
    // All ranks' blocks of this step in this rank's buffer (bounded waits).
    const std::uint32_t* own_flags = p.flags[p.rank] + parity * p.world;
    bool ok = true;
    if (threadIdx.x < p.world) {
        ok = false;
        for (std::uint32_t poll = 0; poll < kFlagPolls; ++poll) {
            if (load_acquire_sys(own_flags + threadIdx.x) == p.step) {
                ok = true;
                break;
            }
            __nanosleep(64);
        }
        if (!ok) flag_error(p.error_word, kErrWaitTimeout);
    }
    if (!__syncthreads_and(ok)) return;
    __threadfence();
    const float* base = p.blocks[p.rank] + static_cast<std::uint64_t>(parity) * p.world * p.block_floats;
    const std::uint32_t warps = blockDim.x / 32;
    for (std::uint64_t row = static_cast<std::uint64_t>(blockIdx.x) * warps + threadIdx.x / 32; row < p.rows;
         row += static_cast<std::uint64_t>(gridDim.x) * warps) {
        lse_merge_row(base, base + p.rows, base + 2 * p.rows, p.world, row, p.head_dim, p.block_floats,
                      p.block_floats, p.block_floats, p.out, threadIdx.x & 31);
    }
}

}  // namespace
}  // namespace ilb

struct InferlabCudaPeerExchange {
    int device = 0;
    std::uint32_t world = 1;
    std::uint32_t rank = 0;
    std::uint64_t rows = 0;
    std::uint32_t head_dim = 0;
    ilb::BufferLayout layout{};
    void* bases[ilb::kMaxRanks] = {};  // receive buffers; peers' opened by IPC
    std::uint32_t* error_word = nullptr;
    std::uint32_t step = 0;
    std::mutex mutex;
};

extern "C" std::uint64_t inferlab_cuda_peer_buffer_bytes(std::uint32_t world, std::uint64_t rows,
                                                         std::uint32_t head_dim) {
    if (world == 0 || world > ilb::kMaxRanks || rows == 0 || head_dim == 0) return 0;
    return ilb::buffer_layout(world, rows, head_dim).bytes;
}

extern "C" int inferlab_cuda_peer_buffer_alloc(int device, std::uint64_t bytes, void** buffer, void* handle,
                                               char* error, std::size_t error_capacity) {
    return ilb::protect(error, error_capacity, [&] {
        if (buffer == nullptr || handle == nullptr || bytes == 0) {
            throw std::runtime_error("peer buffer arguments are invalid");
        }
        ilb::DeviceGuard guard(device);
        void* ptr = nullptr;
        ilb::cuda_check(cudaMalloc(&ptr, bytes), "cudaMalloc peer buffer");
        cudaIpcMemHandle_t h{};
        const cudaError_t zeroed = cudaMemset(ptr, 0, bytes);
        const cudaError_t got = zeroed == cudaSuccess ? cudaIpcGetMemHandle(&h, ptr) : zeroed;
        if (got != cudaSuccess) {
            cudaFree(ptr);
            ilb::cuda_check(got, "peer buffer IPC handle");
        }
        static_assert(sizeof(h) <= INFERLAB_CUDA_IPC_HANDLE_BYTES, "IPC handle size");
        std::memset(handle, 0, INFERLAB_CUDA_IPC_HANDLE_BYTES);
        std::memcpy(handle, &h, sizeof(h));
        *buffer = ptr;
    });
}

extern "C" int inferlab_cuda_peer_buffer_free(int device, void* buffer, char* error,
                                              std::size_t error_capacity) {
    return ilb::protect(error, error_capacity, [&] {
        ilb::DeviceGuard guard(device);
        if (buffer != nullptr) ilb::cuda_check(cudaFree(buffer), "cudaFree peer buffer");
    });
}

extern "C" int inferlab_cuda_peer_exchange_create(int device, std::uint32_t world, std::uint32_t rank,
                                                  std::uint64_t rows, std::uint32_t head_dim,
                                                  void* local_buffer, const void* handles,
                                                  InferlabCudaPeerExchange** out, char* error,
                                                  std::size_t error_capacity) {
    return ilb::protect(error, error_capacity, [&] {
        if (out == nullptr) throw std::runtime_error("peer exchange output pointer is null");
        *out = nullptr;
        if (world == 0 || world > ilb::kMaxRanks || rank >= world) {
            throw std::runtime_error("peer exchange supports 1 to 8 ranks");
        }
        if (rows == 0 || head_dim == 0 || local_buffer == nullptr || (world > 1 && handles == nullptr)) {
            throw std::runtime_error("peer exchange arguments are invalid");
        }
        ilb::DeviceGuard guard(device);
        auto* ex = new InferlabCudaPeerExchange();
        ex->device = device;
        ex->world = world;
        ex->rank = rank;
        ex->rows = rows;
        ex->head_dim = head_dim;
        ex->layout = ilb::buffer_layout(world, rows, head_dim);
        ex->bases[rank] = local_buffer;
        auto fail = [&](cudaError_t status, const char* what) {
            for (std::uint32_t r = 0; r < world; ++r) {
                if (r != rank && ex->bases[r] != nullptr) cudaIpcCloseMemHandle(ex->bases[r]);
            }
            if (ex->error_word != nullptr) cudaFree(ex->error_word);
            delete ex;
            ilb::cuda_check(status, what);
        };
        for (std::uint32_t r = 0; r < world; ++r) {
            if (r == rank) continue;
            cudaIpcMemHandle_t h{};
            std::memcpy(&h, static_cast<const unsigned char*>(handles) + r * INFERLAB_CUDA_IPC_HANDLE_BYTES,
                        sizeof(h));
            void* peer = nullptr;
            const cudaError_t status = cudaIpcOpenMemHandle(&peer, h, cudaIpcMemLazyEnablePeerAccess);
            if (status != cudaSuccess) fail(status, "cudaIpcOpenMemHandle peer buffer");
            ex->bases[r] = peer;
        }
        void* word = nullptr;
        const cudaError_t status = cudaMalloc(&word, 16);
        if (status != cudaSuccess) fail(status, "cudaMalloc peer exchange error word");
        ex->error_word = static_cast<std::uint32_t*>(word);
        const cudaError_t zeroed = cudaMemset(word, 0, 16);
        if (zeroed != cudaSuccess) fail(zeroed, "cudaMemset peer exchange error word");
        *out = ex;
    });
}

extern "C" int inferlab_cuda_peer_exchange_combine(InferlabCudaPeerExchange* exchange, const float* packed,
                                                   float* out, void* stream, char* error,
                                                   std::size_t error_capacity) {
    return ilb::protect(error, error_capacity, [&] {
        if (exchange == nullptr || packed == nullptr || out == nullptr) {
            throw std::runtime_error("peer exchange pointer is null");
        }
        auto& ex = *exchange;
        std::lock_guard<std::mutex> lock(ex.mutex);
        ilb::DeviceGuard guard(ex.device);
        ilb::ExchangeParams p{};
        for (std::uint32_t r = 0; r < ex.world; ++r) {
            auto* base = static_cast<unsigned char*>(ex.bases[r]);
            p.blocks[r] = reinterpret_cast<float*>(base);
            p.flags[r] = reinterpret_cast<std::uint32_t*>(base + ex.layout.flags_offset);
        }
        p.packed = packed;
        p.out = out;
        p.rows = ex.rows;
        p.block_floats = ex.layout.block_floats;
        p.head_dim = ex.head_dim;
        p.world = ex.world;
        p.rank = ex.rank;
        // Steps count from 1 (the zeroed flags match no step); a wrap skips 0.
        if (++ex.step == 0) ex.step = 1;
        p.step = ex.step;
        p.error_word = ex.error_word;
        if (ex.layout.block_floats % 4 == 0 && reinterpret_cast<std::uintptr_t>(packed) % 16 != 0) {
            throw std::runtime_error("peer exchange block must be 16-byte aligned");
        }
        ilb::peer_exchange_kernel<<<ex.world, ilb::kExchangeThreads, 0, static_cast<cudaStream_t>(stream)>>>(p);
        ilb::cuda_check(cudaGetLastError(), "peer exchange launch");
    });
}

extern "C" int inferlab_cuda_peer_exchange_synchronize(InferlabCudaPeerExchange* exchange, void* stream,
                                                       std::uint32_t timeout_ms, char* error,
                                                       std::size_t error_capacity) {
    return ilb::protect(error, error_capacity, [&] {
        if (exchange == nullptr) throw std::runtime_error("peer exchange pointer is null");
        ilb::DeviceGuard guard(exchange->device);
        auto s = static_cast<cudaStream_t>(stream);
        ilb::wait_stream(s, timeout_ms);
        std::uint32_t bits = 0;
        ilb::cuda_check(cudaMemcpy(&bits, exchange->error_word, 4, cudaMemcpyDeviceToHost),
                        "cudaMemcpy peer exchange error word");
        if (bits != 0) {
            ilb::cuda_check(cudaMemset(exchange->error_word, 0, 4), "cudaMemset peer exchange error word");
            throw std::runtime_error(ilb::describe_error_bits(bits));
        }
    });
}

extern "C" void inferlab_cuda_peer_exchange_destroy(InferlabCudaPeerExchange* exchange) {
    if (exchange == nullptr) return;
    {
        int previous = 0;
        cudaGetDevice(&previous);
        cudaSetDevice(exchange->device);
        cudaDeviceSynchronize();
        for (std::uint32_t r = 0; r < exchange->world; ++r) {
            if (r != exchange->rank && exchange->bases[r] != nullptr) cudaIpcCloseMemHandle(exchange->bases[r]);
        }
        if (exchange->error_word != nullptr) cudaFree(exchange->error_word);
        cudaSetDevice(previous);
    }
    delete exchange;
}
