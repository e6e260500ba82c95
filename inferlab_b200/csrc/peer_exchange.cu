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
// library kernel touches peer memory) and merges all ranks' blocks in rank
// order with the same per-row code as inferlab_cuda_lse_combine_packed.
//
// Every element travels as one aligned 8-byte store: its 32 bits in the low
// half, the step number in the high half. An aligned 8-byte store is
// single-copy atomic, so a receiver that reads the current step in a word
// also reads that step's value: no flag and no system-scope fence between
// data and flag. Receive buffer of one rank: words [2 parities][world][rows *
// (D + 2)]. Step s uses parity s & 1: a rank pushes step s + 2 into a peer
// only after its own exchange s + 1 has read that peer's step s + 1 words,
// which the peer wrote only after its exchange s had read its step s words.
#include "common.cuh"
#include "internal.cuh"
#include "lse_merge.cuh"

#include "../../include/inferlab_attention.h"

#include <cstring>
#include <mutex>

namespace ilb {
namespace {

constexpr std::uint32_t kMaxRanks = INFERLAB_CUDA_PEER_MAX_RANKS;
constexpr int kExchangeThreads = 256;
// Bounded wait for the peers' words: 2 s of the GPU's global timer per
// thread, shared by all the words the thread receives.
constexpr unsigned long long kWaitNs = 2000000000ull;

std::uint64_t align256(std::uint64_t n) { return (n + 255) & ~std::uint64_t(255); }

struct BufferLayout {
    std::uint64_t block_floats;  // rows * (head_dim + 2)
    std::uint64_t bytes;
};

BufferLayout buffer_layout(std::uint32_t world, std::uint64_t rows, std::uint32_t head_dim) {
    BufferLayout b{};
    b.block_floats = rows * (static_cast<std::uint64_t>(head_dim) + 2);
    b.bytes = align256(2ull * world * b.block_floats * 8);
    return b;
}

struct ExchangeParams {
    std::uint64_t* words[kMaxRanks];  // every rank's receive words (peer-mapped; own at [rank])
    const float* packed;              // this rank's block
    float* out;
    std::uint64_t rows;
    std::uint64_t block_floats;
    std::uint32_t rows_per_cta;
    std::uint32_t head_dim;
    std::uint32_t world;
    std::uint32_t rank;
    std::uint32_t step;
    std::uint32_t* error_word;
};

__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ std::uint64_t load_word(const std::uint64_t* p) {
    std::uint64_t v;
    asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// CTA c stores this rank's block into rank c's buffer, then receives rows
// [c * R, (c + 1) * R) of every rank's block into shared memory and merges
// them (one warp per row).
__global__ void __launch_bounds__(kExchangeThreads) peer_exchange_kernel(const ExchangeParams p) {
    extern __shared__ float parts[];  // [3][world][R] m, l then [world][R][D] o
    const std::uint32_t parity = p.step & 1u;
    const std::uint64_t tag = static_cast<std::uint64_t>(p.step) << 32;
    {
        std::uint64_t* dst = p.words[blockIdx.x] + (static_cast<std::uint64_t>(parity) * p.world + p.rank) * p.block_floats;
        for (std::uint64_t e = threadIdx.x; e < p.block_floats; e += blockDim.x) {
            dst[e] = tag | __float_as_uint(p.packed[e]);
        }
    }
    const std::uint32_t R = p.rows_per_cta;
    const std::uint64_t r0 = static_cast<std::uint64_t>(blockIdx.x) * R;
    const std::uint64_t left = r0 < p.rows ? p.rows - r0 : 0;  // rows of this CTA
    const std::uint32_t nr = static_cast<std::uint32_t>(left < R ? left : R);
    float* sm_m = parts;
    float* sm_l = parts + p.world * R;
    float* sm_o = parts + 2 * p.world * R;
    const std::uint64_t* own = p.words[p.rank] + static_cast<std::uint64_t>(parity) * p.world * p.block_floats;
    // Per source rank, this CTA's rows: nr m words, nr l words, nr * D o words.
    const std::uint32_t per_src = nr * (p.head_dim + 2);
    // Each thread takes its words eight at a time: the eight loads are in
    // flight together, and only the words not yet of this step are polled
    // again.
    constexpr int kBatch = 8;
    const std::uint32_t total = p.world * per_src;
    const unsigned long long deadline = global_ns() + kWaitNs;
    bool ok = true;
    for (std::uint32_t base = threadIdx.x; ok && base < total; base += kBatch * blockDim.x) {
        const std::uint64_t* w[kBatch];
        float* slot[kBatch];
        std::uint64_t v[kBatch];
        bool need[kBatch];
#pragma unroll
        for (int u = 0; u < kBatch; ++u) {
            const std::uint32_t j = base + u * blockDim.x;
            need[u] = j < total;
            w[u] = own;
            slot[u] = sm_m;
            if (!need[u]) continue;
            const std::uint32_t src = j / per_src;
            const std::uint32_t i = j % per_src;
            std::uint64_t e;
            if (i < nr) {
                e = r0 + i;
                slot[u] = sm_m + src * R + i;
            } else if (i < 2 * nr) {
                e = p.rows + r0 + (i - nr);
                slot[u] = sm_l + src * R + (i - nr);
            } else {
                const std::uint32_t k = i - 2 * nr;
                e = 2 * p.rows + r0 * p.head_dim + k;  // rows r0.. are contiguous in the o block
                slot[u] = sm_o + (static_cast<std::uint64_t>(src) * R) * p.head_dim + k;
            }
            w[u] = own + static_cast<std::uint64_t>(src) * p.block_floats + e;
        }
#pragma unroll
        for (int u = 0; u < kBatch; ++u) v[u] = need[u] ? load_word(w[u]) : 0;
        for (;;) {
            bool waiting = false;
#pragma unroll
            for (int u = 0; u < kBatch; ++u) {
                if (!need[u]) continue;
                if ((v[u] & 0xFFFFFFFF00000000ull) == tag) {
                    *slot[u] = __uint_as_float(static_cast<std::uint32_t>(v[u]));
                    need[u] = false;
                } else {
                    waiting = true;
                }
            }
            if (!waiting) break;
            if (global_ns() > deadline) {
                ok = false;
                break;
            }
            __nanosleep(64);
#pragma unroll
            for (int u = 0; u < kBatch; ++u) {
                if (need[u]) v[u] = load_word(w[u]);
            }
        }
    }
    if (!ok) flag_error(p.error_word, kErrWaitTimeout);
    if (!__syncthreads_and(ok)) return;
    const std::uint32_t warps = blockDim.x / 32;
    for (std::uint32_t k = threadIdx.x / 32; k < nr; k += warps) {
        lse_merge_row(sm_m, sm_l, sm_o, p.world, k, p.head_dim, R, R,
                      static_cast<std::uint64_t>(R) * p.head_dim, p.out + r0 * p.head_dim, threadIdx.x & 31);
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

namespace ilb {

ExchangeView exchange_take_step(InferlabCudaPeerExchange* exchange, int device, std::uint64_t rows,
                                std::uint32_t head_dim) {
    if (exchange == nullptr) throw std::runtime_error("peer exchange pointer is null");
    auto& ex = *exchange;
    std::lock_guard<std::mutex> lock(ex.mutex);
    if (ex.device != device || ex.rows != rows || ex.head_dim != head_dim) {
        throw std::runtime_error("peer exchange does not match the decode batch");
    }
    ExchangeView v{};
    for (std::uint32_t r = 0; r < ex.world; ++r) v.words[r] = static_cast<std::uint64_t*>(ex.bases[r]);
    v.world = ex.world;
    v.rank = ex.rank;
    if (++ex.step == 0) ex.step = 1;  // the zeroed words carry step 0
    v.step = ex.step;
    v.rows = ex.rows;
    v.head_dim = ex.head_dim;
    v.device = ex.device;
    return v;
}

}  // namespace ilb

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
        for (std::uint32_t r = 0; r < ex.world; ++r) p.words[r] = static_cast<std::uint64_t*>(ex.bases[r]);
        p.packed = packed;
        p.out = out;
        p.rows = ex.rows;
        p.block_floats = ex.layout.block_floats;
        p.rows_per_cta = static_cast<std::uint32_t>((ex.rows + ex.world - 1) / ex.world);
        p.head_dim = ex.head_dim;
        p.world = ex.world;
        p.rank = ex.rank;
        p.error_word = ex.error_word;
        const std::size_t smem = static_cast<std::size_t>(ex.world) * p.rows_per_cta * (ex.head_dim + 2) * 4;
        if (smem > 200 * 1024) throw std::runtime_error("peer exchange rows do not fit a CTA");
        // Steps count from 1 (the zeroed words carry step 0); a wrap skips 0.
        // The step is taken only once the call can launch, so a rejected call
        // leaves this rank's count in step with its peers'.
        if (++ex.step == 0) ex.step = 1;
        p.step = ex.step;
        ilb::cuda_check(cudaFuncSetAttribute(ilb::peer_exchange_kernel,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)),
                        "cudaFuncSetAttribute");
        ilb::peer_exchange_kernel<<<ex.world, ilb::kExchangeThreads, smem, static_cast<cudaStream_t>(stream)>>>(p);
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
