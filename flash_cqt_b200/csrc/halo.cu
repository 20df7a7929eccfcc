// Overlap-add halo of the slice-range partitioned sliced transform, over
// peer memory (NVLink / NVSwitch), no collective library on the data path.
//
// Rank r owns slices [s0, s1) of a long stream; its synthesis overlap-adds
// into one hop before its owned samples plus the owned samples, and that
// first hop belongs to rank r - 1 (its last owned hop also receives the
// first-half terms of rank r's first slice).  So every rank r > 0 sends one
// hop (rows x hop floats) to rank r - 1, which adds it in.
//
// Each rank allocates one exchange buffer and exports it by CUDA IPC:
//   [0]    data flag: the epoch of the hop that sits in the buffer (written
//          by the right neighbour after its data)
//   [8]    ack flag: the last epoch the left neighbour has consumed from the
//          buffer this rank writes into (written by the left neighbour)
//   [128]  rows x hop floats of received data
// Send (rank r, into rank r - 1's buffer): wait until rank r - 1 has consumed
// the previous epoch (ack in r's own buffer), store the hop with plain peer
// stores, and once every CTA has fenced its stores at system scope, the last
// CTA raises the neighbour's data flag to the epoch with a system-scope
// release.  Receive (rank r - 1): wait for its own data flag to reach the
// epoch (system-scope acquire), add the hop into its output, and the last CTA
// acknowledges by writing the epoch into rank r's ack flag.  Every wait polls the global
// timer and gives up after the exchange's limit (10 s unless set), counting
// itself in the exchange's
// status word (the host reads it; nothing hangs), and a send or receive that
// gave up skips its data movement.  No multicast object, no NVLS: a rank
// that dies leaves its neighbours with expired waits, not with faults.
#include <cstdint>
#include <cstring>

#include <cuda_runtime.h>

#include "internal.h"

namespace fcqt {

namespace {

constexpr size_t kHaloHeader = 128;

__device__ __forceinline__ unsigned long long now_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ long long load_acquire_sys(const long long* p) {
    long long v;
    asm volatile("ld.acquire.sys.global.s64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void store_release_sys(long long* p, long long v) {
    asm volatile("st.release.sys.global.s64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// one thread per CTA waits until *flag >= want (bounded); the CTA learns the
// outcome through shared memory.  A wait that gives up counts itself in the
// status word and marks the epoch failed.
__device__ bool cta_wait_flag(const long long* flag, long long want, unsigned* status,
                              long long* failed, long long epoch, unsigned long long limit_ns) {
    __shared__ int ok;
    if (threadIdx.x == 0) {
        ok = 1;
        if (load_acquire_sys(flag) < want) {
            const unsigned long long t0 = now_ns();
            while (load_acquire_sys(flag) < want) {
                if (now_ns() - t0 > limit_ns) {
                    ok = 0;
                    atomicAdd(status, 1u);
                    atomicExch(reinterpret_cast<unsigned long long*>(failed),
                               (unsigned long long)epoch);
                    break;
                }
                __nanosleep(256);
            }
        }
    }
    __syncthreads();
    return ok != 0;
}

// the last CTA of the grid to finish publishes `epoch` to a peer's flag with
// a system-scope release -- after every CTA has fenced its own stores at
// system scope -- unless some CTA marked the epoch failed
__device__ void last_cta_publish(unsigned* counter, long long* peer_flag, long long epoch,
                                 const long long* failed) {
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned nblocks = gridDim.x * gridDim.y;
        if (atomicAdd(counter, 1u) == nblocks - 1) {
            *counter = 0;   // ready for the next epoch (stream-ordered)
            __threadfence_system();
            if (*reinterpret_cast<const volatile long long*>(failed) != epoch)
                store_release_sys(peer_flag, epoch);
        }
    }
}

}  // namespace

struct HaloDev {       // device words of one exchange (own memory)
    unsigned status;   // expired waits
    unsigned send_done, recv_done;   // CTA counters of the last-CTA pattern
    unsigned pad;
    long long send_failed, recv_failed;   // last epoch whose wait gave up
};

namespace {

// rows x hop floats src (row stride ld) -> the left neighbour's data area
// (dense), then its data flag := epoch
__global__ void __launch_bounds__(256)
halo_send_kernel(const float* __restrict__ src, long long ld, long long hop,
                 char* __restrict__ left, const long long* own_ack, long long epoch,
                 HaloDev* dv, unsigned long long limit_ns) {
    if (cta_wait_flag(own_ack, epoch - 1, &dv->status, &dv->send_failed, epoch, limit_ns)) {
        const long long row = blockIdx.y;
        const float* s = src + row * ld;
        float* d = reinterpret_cast<float*>(left + 128) + row * hop;
        for (long long i = blockIdx.x * 256LL + threadIdx.x; i < hop; i += 256LL * gridDim.x)
            d[i] = s[i];
    }
    last_cta_publish(&dv->send_done, reinterpret_cast<long long*>(left), epoch,
                     &dv->send_failed);
}

// wait for the own data flag to reach epoch, dst += the received hop, then the
// right neighbour's ack flag := epoch (its buffer here is free again)
__global__ void __launch_bounds__(256)
halo_recv_kernel(float* __restrict__ dst, long long ld, long long hop,
                 const char* __restrict__ own, char* right, long long epoch, HaloDev* dv,
                 unsigned long long limit_ns) {
    if (cta_wait_flag(reinterpret_cast<const long long*>(own), epoch, &dv->status,
                      &dv->recv_failed, epoch, limit_ns)) {
        const long long row = blockIdx.y;
        float* d = dst + row * ld;
        const float* s = reinterpret_cast<const float*>(own + 128) + row * hop;
        for (long long i = blockIdx.x * 256LL + threadIdx.x; i < hop; i += 256LL * gridDim.x)
            d[i] += s[i];
    }
    last_cta_publish(&dv->recv_done, reinterpret_cast<long long*>(right + 8), epoch,
                     &dv->recv_failed);
}

}  // namespace

size_t halo_buffer_bytes(int rows, long long hop) {
    return kHaloHeader + (size_t)rows * (size_t)hop * sizeof(float);
}

cudaError_t halo_create(HaloState* h, void* handle_out) {
    h->own = nullptr;
    h->dv = nullptr;
    cudaError_t e = cudaMalloc(&h->own, halo_buffer_bytes(h->rows, h->hop));
    if (e != cudaSuccess) return e;
    e = cudaMemset(h->own, 0, kHaloHeader);   // both flags at epoch 0
    if (e == cudaSuccess) e = cudaMalloc(&h->dv, sizeof(HaloDev));
    if (e == cudaSuccess) e = cudaMemset(h->dv, 0, sizeof(HaloDev));
    cudaIpcMemHandle_t ih;
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&ih, h->own);
    if (e == cudaSuccess) std::memcpy(handle_out, &ih, sizeof ih);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();   // flags are zero before any peer looks
    return e;
}

cudaError_t halo_open(const void* handle, char** out) {
    cudaIpcMemHandle_t ih;
    std::memcpy(&ih, handle, sizeof ih);
    void* p = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&p, ih, cudaIpcMemLazyEnablePeerAccess);
    *out = static_cast<char*>(p);
    return e;
}

dim3 halo_grid(const HaloState* h) {
    return dim3((unsigned)((h->hop + 256 * 8 - 1) / (256 * 8)), (unsigned)h->rows);
}

cudaError_t halo_send(HaloState* h, const float* src, long long ld, long long epoch,
                      cudaStream_t s) {
    halo_send_kernel<<<halo_grid(h), 256, 0, s>>>(src, ld, h->hop, h->left,
                                                  reinterpret_cast<const long long*>(h->own + 8),
                                                  epoch, h->dv, h->wait_ns);
    return cudaGetLastError();
}

cudaError_t halo_recv_add(HaloState* h, float* dst, long long ld, long long epoch,
                          cudaStream_t s) {
    halo_recv_kernel<<<halo_grid(h), 256, 0, s>>>(dst, ld, h->hop, h->own, h->right, epoch,
                                                  h->dv, h->wait_ns);
    return cudaGetLastError();
}

cudaError_t halo_status(HaloState* h, unsigned* expired, int clear) {
    cudaError_t e = cudaMemcpy(expired, &h->dv->status, sizeof(unsigned), cudaMemcpyDeviceToHost);
    if (e == cudaSuccess && clear) e = cudaMemset(&h->dv->status, 0, sizeof(unsigned));
    return e;
}

void halo_destroy(HaloState* h) {
    if (h->left) cudaIpcCloseMemHandle(h->left);
    if (h->right) cudaIpcCloseMemHandle(h->right);
    if (h->own) cudaFree(h->own);
    if (h->dv) cudaFree(h->dv);
}

}  // namespace fcqt
