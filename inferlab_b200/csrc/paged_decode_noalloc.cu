// paged_decode_noalloc.cu - paged decode for callers that cannot allocate.
//
// inferlab_cuda_paged_decode takes its split-KV scratch from the caller (a
// workspace the caller allocates once). Some callers cannot hand one over:
// a host process whose device memory is reserved up front by another
// framework's caching allocator, or a serving loop that may not call
// cudaMalloc (with its implicit device synchronisation) once it is running.
// For them this entry point keeps the scratch in a fixed array compiled into
// the library: a file-scope __device__ array of kStaticScratchBytes, which
// every GPU that loads this part of the library holds until the process
// exits. It allocates nothing itself (no cudaMalloc, cudaFree or allocating
// library call); the caller still passes the queries, tables and output.
//
// The array is shared by every call on a device and keeps the last call's
// contents, so each call first clears the split counters at its front; two
// calls whose work overlaps on the GPU (different streams, or different
// host threads on one device) race on the array and must be serialised by
// the caller. Batches whose contexts all fit one split need no scratch and
// never touch the array. The first call on a device that needs scratch looks
// up the array's device address (cudaGetSymbolAddress with that device
// current) and caches it for the life of the process; make that first call
// before any stream capture. A device reset (cudaDeviceReset, or a context
// torn down and created again on that device) reloads the library's module
// and leaves the cached address stale, so calls after one are not supported.
#include "common.cuh"
#include "internal.cuh"
#include "pool.cuh"

#include "../../include/inferlab_attention.h"

#include <mutex>
#include <string>

namespace {

constexpr std::size_t kStaticScratchBytes = std::size_t(16) << 20;  // 16 MiB

static __device__ __align__(256) unsigned char g_decode_scratch[kStaticScratchBytes];

std::mutex g_scratch_mutex;
void* g_scratch_address[128] = {};

// Device address of g_decode_scratch on `device`, which must be current. The
// host-side name of the array is only a stand-in: it must never be passed to a
// kernel, only the address this returns.
void* scratch_address(int device) {
    if (device < 0 || device >= 128) throw std::runtime_error("CUDA device index out of range");
    std::lock_guard<std::mutex> lock(g_scratch_mutex);
    if (g_scratch_address[device] == nullptr) {
        void* address = nullptr;
        ilb::cuda_check(cudaGetSymbolAddress(&address, g_decode_scratch),
                        "cudaGetSymbolAddress(decode scratch)");
        g_scratch_address[device] = address;
    }
    return g_scratch_address[device];
}

}  // namespace

extern "C" int inferlab_cuda_paged_decode_noalloc(InferlabCudaKvPool* pool, const float* queries,
                                                  const std::int32_t* block_tables,
                                                  std::uint32_t max_blocks_per_seq,
                                                  const std::int32_t* context_lens,
                                                  std::uint32_t num_seqs, std::uint32_t q_heads,
                                                  std::uint32_t max_context_len, float* out,
                                                  void* stream, char* error,
                                                  std::size_t error_capacity) {
    return ilb::protect(error, error_capacity, [&] {
        using namespace ilb;
        auto& p = checked_pool(pool);
        if (num_seqs == 0) return;
        check_decode_arguments(p, queries, block_tables, max_blocks_per_seq, context_lens,
                               num_seqs, q_heads, max_context_len);
        if (out == nullptr) throw std::runtime_error("paged decode output pointer is null");
        // Only a batch whose contexts are split across CTAs keeps partials in
        // scratch; one split per sequence (or the generic kernel) reads none.
        const std::size_t need = decode_scratch_bytes(p, num_seqs, q_heads, max_context_len);
        if (need > kStaticScratchBytes) {
            throw std::runtime_error(
                "paged decode batch needs " + std::to_string(need) +
                " bytes of scratch, more than the 16777216 built into the allocation-free entry "
                "point; use inferlab_cuda_paged_decode with a caller workspace");
        }
        DeviceGuard guard(p.device);
        auto s = static_cast<cudaStream_t>(stream);
        void* scratch = nullptr;
        if (need > 0) {
            scratch = scratch_address(p.device);
            // The split counters must start at zero; the rest is written before it is read.
            cuda_check(cudaMemsetAsync(scratch, 0, decode_counter_bytes(p, num_seqs), s),
                       "cudaMemsetAsync(decode scratch counters)");
        }
        launch_paged_decode(p, queries, block_tables, max_blocks_per_seq, context_lens, num_seqs,
                            q_heads, max_context_len, out, scratch,
                            scratch != nullptr ? kStaticScratchBytes : 0, s);
    });
}
