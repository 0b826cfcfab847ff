// xchg.cu -- rank-to-rank all-gather over NVLink for the column-split vocab head.
//
// The split head exchanges two small arrays per token step (every rank's hidden-state
// rows before the head, every rank's per-row (max, index, exp-sum) parts after it).
// At these sizes (tens of KB) a collective library's all-gather is latency-bound, and
// concurrent decoders serialise on it.  Here each rank owns one device buffer that its
// peers map through CUDA IPC:
//
//   [0, 256)          flags: u64 flags[r] = sequence number of rank r's last call,
//                     written by rank r; u64 at byte 128: this rank's call counter
//   [256, ...)        data[parity][rank][cap]: rank r's rows of call s at parity s & 1
//
// One launch per all-gather, one CTA: thread 0 advances the call counter (every rank
// makes the same calls in the same order, so the counters agree); all threads store
// the caller's rows into data[s & 1][rank] of every rank's buffer (peer stores over
// NVLink); a system-scope fence; thread 0 publishes s in every rank's flags[rank]
// (st.release.sys), then waits -- bounded -- until every flags[r] of its own buffer
// reaches s (ld.acquire.sys); the CTA then copies data[s & 1][0 .. world) to the
// caller's output, rank-major.  Call s + 2 rewrites the parity of call s only after
// every peer has published s + 1, i.e. after each peer's call s has finished reading.
// A wait that expires (~30 s) records kDevErrWaitTimeout and returns (no trap, no hang).
// Ranks must run on distinct GPUs (the Python layer checks), so the waiting kernels
// never share a GPU.
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include "common.cuh"
#include "internal.h"

namespace madi {
namespace {

constexpr int kXThreads = 512;
constexpr size_t kXHeader = 256;
// The wait for the peers' flags: ~30 s at 2 GHz.  Longer than the kernels' usual
// budget because ranks can drift apart by seconds before their first exchange (each
// captures its graphs and loads its modules on its own schedule); still finite.
constexpr long long kXchgWaitCycles = 60000000000LL;

struct PeerBases {
    uint8_t *base[kXchgMaxWorld];     // every rank's buffer, as this rank maps it
};

MADI_DEV void st_release_sys(uint64_t *p, uint64_t v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
MADI_DEV uint64_t ld_acquire_sys(const uint64_t *p) {
    uint64_t v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__global__ void __launch_bounds__(kXThreads) xchg_allgather_kernel(PeerBases peers, int world, int rank, size_t cap,
                                                                   const uint4 *__restrict__ src, int nvec,
                                                                   uint4 *__restrict__ dst, int *dev_err) {
    __shared__ uint64_t s_seq;
    __shared__ int s_ok;
    uint8_t *mine = peers.base[rank];
    if (threadIdx.x == 0) {
        uint64_t *counter = reinterpret_cast<uint64_t *>(mine + 128);
        s_seq = *counter + 1;
        *counter = s_seq;
        s_ok = 1;
    }
    __syncthreads();
    const uint64_t seq = s_seq;
    const size_t slot = ((size_t)(seq & 1) * world + rank) * cap;
    for (int r = 0; r < world; ++r) {
        uint4 *to = reinterpret_cast<uint4 *>(peers.base[r] + kXHeader + slot);
        for (int i = threadIdx.x; i < nvec; i += blockDim.x) to[i] = src[i];
    }
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int r = 0; r < world; ++r) st_release_sys(reinterpret_cast<uint64_t *>(peers.base[r]) + rank, seq);
        const uint64_t *flags = reinterpret_cast<const uint64_t *>(mine);
        const long long t0 = clock64();
        for (int r = 0; r < world && s_ok; ++r) {
            while (ld_acquire_sys(flags + r) < seq) {
                if (clock64() - t0 > kXchgWaitCycles) {
                    if (dev_err) atomicCAS(dev_err, kDevErrNone, kDevErrWaitTimeout);
                    s_ok = 0;
                    break;
                }
            }
        }
    }
    __syncthreads();
    if (!s_ok) return;
    // the peers' rows, read past the L1 (they arrived over NVLink after this CTA's
    // acquire of their flags)
    const size_t row = cap / 16;
    const uint4 *from = reinterpret_cast<const uint4 *>(mine + kXHeader + (size_t)(seq & 1) * world * cap);
    for (int r = 0; r < world; ++r)
        for (int i = threadIdx.x; i < nvec; i += blockDim.x) dst[(size_t)r * nvec + i] = __ldcv(from + (size_t)r * row + i);
}

}  // namespace

size_t xchg_buffer_bytes(int world, size_t cap) { return kXHeader + 2 * (size_t)world * cap; }

cudaError_t launch_xchg_allgather(uint8_t *const *bases, int world, int rank, size_t cap, const void *src,
                                  size_t bytes, void *dst, int *dev_err, cudaStream_t st) {
    PeerBases pb;
    memset(&pb, 0, sizeof(pb));
    for (int r = 0; r < world; ++r) pb.base[r] = bases[r];
    xchg_allgather_kernel<<<1, kXThreads, 0, st>>>(pb, world, rank, cap, static_cast<const uint4 *>(src),
                                                   (int)(bytes / 16), static_cast<uint4 *>(dst), dev_err);
    return cudaGetLastError();
}

}  // namespace madi
