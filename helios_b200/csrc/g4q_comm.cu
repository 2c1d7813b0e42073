// g4q_comm.cu -- tensor-parallel allreduce(sum) over NVLink peer memory, bounded waits.
//
// The TP communicator of the hot path's boundary: the sum after o_proj and down_proj when the
// linears are sharded (the reference runs one process per model and has no collective; its
// sharded equivalent is the Megatron split of the same linears). One process per GPU; every rank
// owns an exchange buffer that the other ranks map through CUDA IPC and write with plain peer
// stores (no multicast, no library kernel on peer memory).
//
//  * Small messages (<= 256 KB): one shot. Every rank pushes its whole vector into its slot of
//    every rank's buffer, then sums the ranks' slots in rank order.
//  * Large messages: two shots. Rank s owns slice s (chunk aligned); every rank pushes slice s of
//    its vector to rank s only, rank s sums its slice over the ranks in rank order and pushes the
//    result to every rank, every rank copies the gathered result back. NVLink traffic per rank is
//    2 (n-1)/n of the vector instead of (n-1) times it.
//
// Each 4096-element chunk is published by a flag word written with st.release.sys after the
// chunk's stores (CTA barrier + system fence first); readers acquire the flag, then read through
// L2. Flags carry a tag unique per call (a device-side call counter, so CUDA-graph replays stay
// correct), and slots alternate between two buffers by call parity: a rank can be at most one call
// ahead of another, because finishing a call needs every rank's contribution to it. Sums run in
// fp32 in rank order, so every rank gets the same bits. Every wait is bounded: a wait that gives up
// records code 40 in the device error word and the kernel runs to its end (results invalid).
#include <cstring>
#include <string>

#include "g4q_common.cuh"
#include "g4q_internal.h"

namespace g4q {
namespace {

constexpr int kCommThreads = 512;
constexpr int64_t kChunk = 4096;                    // elements per published chunk
constexpr int64_t kOneShotBytes = 256 * 1024;       // larger messages take two shots
constexpr long long kCommSpinLimit = 4000000000ll;  // ~2 s of SM clocks
constexpr uint64_t kCommMagic = 0x47345143434f4d4dull;

struct ArArgs {
    void* data;
    int64_t count;
    int esize;  // 2 (bf16) or 4 (fp32)
    int rank, n_ranks;
    int two_shot;
    int64_t slot_bytes;   // bytes of one rank slot (= the capacity in fp32 elements x 4)
    int64_t fc;           // flag words per (parity, rank)
    char* const* peers;   // [n_ranks] exchange buffers (own included)
    unsigned int* state;  // [0] calls so far, [1] exit counter
    int* err;
};

// exchange-buffer layout: slots [2][R][slot_bytes], results [2][slot_bytes], flags [2][R][fc],
// result flags [2][fc] (uint32)
__device__ __forceinline__ int64_t slot_off(const ArArgs& a, int par, int r) {
    return ((int64_t)par * a.n_ranks + r) * a.slot_bytes;
}
__device__ __forceinline__ int64_t result_off(const ArArgs& a, int par) {
    return (int64_t)2 * a.n_ranks * a.slot_bytes + (int64_t)par * a.slot_bytes;
}
__device__ __forceinline__ int64_t flag_off(const ArArgs& a, int par, int r, int64_t ch) {
    return (int64_t)2 * (a.n_ranks + 1) * a.slot_bytes + (((int64_t)par * a.n_ranks + r) * a.fc + ch) * 4;
}
__device__ __forceinline__ int64_t rflag_off(const ArArgs& a, int par, int64_t ch) {
    return (int64_t)2 * (a.n_ranks + 1) * a.slot_bytes +
           ((int64_t)2 * a.n_ranks * a.fc + (int64_t)par * a.fc + ch) * 4;
}

__device__ __forceinline__ void st_release_sys(unsigned int* p, unsigned int v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned int ld_acquire_sys(const unsigned int* p) {
    unsigned int v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// one thread: wait until *p == tag (bounded); false when this or another wait gave up
__device__ bool wait_tag(const unsigned int* p, unsigned int tag, int* err) {
    if (ld_acquire_sys(p) == tag) return true;
    const long long t0 = clock64();
    while (ld_acquire_sys(p) != tag) {
        if (*reinterpret_cast<volatile int*>(err) != 0) return false;
        if (clock64() - t0 > kCommSpinLimit) {
            atomicCAS(err, 0, 40);
            return false;
        }
        __nanosleep(64);
    }
    return true;
}

// the whole CTA: copy `bytes` (multiple of 16) from src to dst
__device__ __forceinline__ void copy16(char* dst, const char* src, int64_t bytes) {
    for (int64_t i = threadIdx.x; i < bytes / 16; i += blockDim.x)
        reinterpret_cast<uint4*>(dst)[i] = __ldcg(reinterpret_cast<const uint4*>(src) + i);
}

// the whole CTA: publish `tag` in every listed flag word after the CTA's stores
__device__ __forceinline__ void publish(unsigned int* const* flags, int n, unsigned int tag) {
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        for (int i = 0; i < n; ++i) st_release_sys(flags[i], tag);
    }
    __syncthreads();   // the flag list may be rewritten for the next chunk only after this
}

// out[i] = sum over ranks (rank order, fp32) of slot r element i, for elements [lo, lo + n)
__device__ __forceinline__ void reduce_chunk(const ArArgs& a, const char* own, int par, int64_t lo, int64_t n,
                                             char* out) {
    if (a.esize == 4) {
        for (int64_t i = threadIdx.x; i < n / 4; i += blockDim.x) {
            float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int r = 0; r < a.n_ranks; ++r) {
                const float4 v = __ldcg(reinterpret_cast<const float4*>(own + slot_off(a, par, r) + lo * 4) + i);
                s.x += v.x;
                s.y += v.y;
                s.z += v.z;
                s.w += v.w;
            }
            reinterpret_cast<float4*>(out + lo * 4)[i] = s;
        }
    } else {
        for (int64_t i = threadIdx.x; i < n / 8; i += blockDim.x) {
            float s[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
            for (int r = 0; r < a.n_ranks; ++r) {
                const uint4 v = __ldcg(reinterpret_cast<const uint4*>(own + slot_off(a, par, r) + lo * 2) + i);
                const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    s[2 * e] += bf16_bits_to_f32(w[e] & 0xffffu);
                    s[2 * e + 1] += bf16_bits_to_f32(w[e] >> 16);
                }
            }
            uint4 o;
            o.x = (uint32_t)f32_to_bf16_bits(s[0]) | ((uint32_t)f32_to_bf16_bits(s[1]) << 16);
            o.y = (uint32_t)f32_to_bf16_bits(s[2]) | ((uint32_t)f32_to_bf16_bits(s[3]) << 16);
            o.z = (uint32_t)f32_to_bf16_bits(s[4]) | ((uint32_t)f32_to_bf16_bits(s[5]) << 16);
            o.w = (uint32_t)f32_to_bf16_bits(s[6]) | ((uint32_t)f32_to_bf16_bits(s[7]) << 16);
            reinterpret_cast<uint4*>(out + lo * 2)[i] = o;
        }
    }
}

// first element of slice s (chunk aligned; the last slice takes the rest)
__device__ __forceinline__ int64_t slice_lo(int64_t count, int s, int R) {
    if (s >= R) return count;
    const int64_t nch = (count + kChunk - 1) / kChunk;
    return (nch * s / R) * kChunk;
}

__global__ void __launch_bounds__(kCommThreads, 1) allreduce_kernel(ArArgs a) {
    __shared__ unsigned int s_tag;
    __shared__ int s_ok;
    __shared__ unsigned int* s_flags[8];
    if (threadIdx.x == 0) {
        const unsigned int calls = *reinterpret_cast<volatile unsigned int*>(a.state);
        s_tag = calls % 0xFFFFFFFEu + 1u;   // never 0 (the value flags start with)
    }
    __syncthreads();
    const unsigned int tag = s_tag;
    const int par = (int)((tag - 1u) & 1u);
    const int R = a.n_ranks;
    char* own = a.peers[a.rank];
    char* data = reinterpret_cast<char*>(a.data);
    const int64_t nch = (a.count + kChunk - 1) / kChunk;
    auto chunk_n = [&](int64_t ch) { return (ch + 1) * kChunk <= a.count ? kChunk : a.count - ch * kChunk; };

    if (!a.two_shot) {
        // push my vector into my slot of every rank's buffer
        for (int64_t ch = blockIdx.x; ch < nch; ch += gridDim.x) {
            const int64_t lo = ch * kChunk, bytes = chunk_n(ch) * a.esize;
            for (int p = 0; p < R; ++p)
                copy16(a.peers[p] + slot_off(a, par, a.rank) + lo * a.esize, data + lo * a.esize, bytes);
            if (threadIdx.x < R)
                s_flags[threadIdx.x] = reinterpret_cast<unsigned int*>(a.peers[threadIdx.x] + flag_off(a, par, a.rank, ch));
            publish(s_flags, R, tag);
        }
        // sum the ranks' slots in rank order
        for (int64_t ch = blockIdx.x; ch < nch; ch += gridDim.x) {
            if (threadIdx.x == 0) {
                int ok = 1;
                for (int r = 0; r < R && ok; ++r)
                    ok = wait_tag(reinterpret_cast<const unsigned int*>(own + flag_off(a, par, r, ch)), tag, a.err);
                s_ok = ok;
            }
            __syncthreads();
            if (s_ok) reduce_chunk(a, own, par, ch * kChunk, chunk_n(ch), data);
            __syncthreads();
        }
    } else {
        // shot 1: slice s of my vector to rank s
        for (int64_t ch = blockIdx.x; ch < nch; ch += gridDim.x) {
            int s = 0;
            while (s + 1 < R && slice_lo(a.count, s + 1, R) <= ch * kChunk) ++s;
            const int64_t lo = ch * kChunk, bytes = chunk_n(ch) * a.esize;
            copy16(a.peers[s] + slot_off(a, par, a.rank) + lo * a.esize, data + lo * a.esize, bytes);
            if (threadIdx.x == 0) s_flags[0] = reinterpret_cast<unsigned int*>(a.peers[s] + flag_off(a, par, a.rank, ch));
            publish(s_flags, 1, tag);
        }
        // reduce my slice; push the result to every rank
        const int64_t mlo = slice_lo(a.count, a.rank, R) / kChunk;
        const int64_t mhi = (slice_lo(a.count, a.rank + 1, R) + kChunk - 1) / kChunk;
        for (int64_t ch = mlo + blockIdx.x; ch < mhi; ch += gridDim.x) {
            if (threadIdx.x == 0) {
                int ok = 1;
                for (int r = 0; r < R && ok; ++r)
                    ok = wait_tag(reinterpret_cast<const unsigned int*>(own + flag_off(a, par, r, ch)), tag, a.err);
                s_ok = ok;
            }
            __syncthreads();
            const int64_t lo = ch * kChunk, n = chunk_n(ch);
            if (s_ok) {
                reduce_chunk(a, own, par, lo, n, own + result_off(a, par));
                __syncthreads();
                for (int p = 0; p < R; ++p)
                    if (p != a.rank)
                        copy16(a.peers[p] + result_off(a, par) + lo * a.esize, own + result_off(a, par) + lo * a.esize,
                               n * a.esize);
            }
            if (threadIdx.x < R)
                s_flags[threadIdx.x] = reinterpret_cast<unsigned int*>(a.peers[threadIdx.x] + rflag_off(a, par, ch));
            publish(s_flags, R, tag);
        }
        // shot 2 received: copy the gathered result back
        for (int64_t ch = blockIdx.x; ch < nch; ch += gridDim.x) {
            if (threadIdx.x == 0)
                s_ok = wait_tag(reinterpret_cast<const unsigned int*>(own + rflag_off(a, par, ch)), tag, a.err) ? 1 : 0;
            __syncthreads();
            const int64_t lo = ch * kChunk;
            if (s_ok) copy16(data + lo * a.esize, own + result_off(a, par) + lo * a.esize, chunk_n(ch) * a.esize);
            __syncthreads();
        }
    }
    // the last CTA out advances the call counter
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        if (atomicAdd(a.state + 1, 1u) == gridDim.x - 1) {
            atomicExch(a.state + 1, 0u);
            atomicAdd(a.state, 1u);
        }
    }
}

struct Comm {
    uint64_t magic = 0;
    int device = -1;
    int rank = 0, n_ranks = 1;
    int64_t max_elems = 0, slot_bytes = 0, fc = 0;
    size_t buf_bytes = 0;
    char* d_buf = nullptr;
    char* peer[8] = {};
    char** d_peers = nullptr;
    unsigned int* d_state = nullptr;
    bool peers_set = false;
};

Comm* checked_comm(const void* h) {
    auto* c = static_cast<Comm*>(const_cast<void*>(h));
    if (!c || c->magic != kCommMagic) throw Error(G4Q_ERR_INVALID_ARGUMENT, "invalid communicator handle");
    return c;
}

void free_comm(Comm* c) {
    cudaFree(c->d_buf);
    cudaFree(c->d_peers);
    cudaFree(c->d_state);
}

}  // namespace

void* comm_create(int rank, int n_ranks, int64_t max_elems) {
    if (n_ranks < 1 || n_ranks > 8 || rank < 0 || rank >= n_ranks)
        throw Error(G4Q_ERR_INVALID_ARGUMENT, "rank must be in [0, n_ranks) with 1 <= n_ranks <= 8");
    if (max_elems <= 0 || max_elems > (1ll << 31))
        throw Error(G4Q_ERR_INVALID_ARGUMENT, "max_elems must be in [1, 2^31]");
    (void)device_scratch();   // the device error word the allreduce's bounded waits report into
    Comm* c = new (std::nothrow) Comm();
    if (!c) throw Error(G4Q_ERR_MEMORY_GUARD, "host allocation failed");
    c->device = current_device();
    c->rank = rank;
    c->n_ranks = n_ranks;
    c->max_elems = (max_elems + kChunk - 1) / kChunk * kChunk;
    c->slot_bytes = c->max_elems * 4;
    c->fc = c->max_elems / kChunk;
    c->buf_bytes = (size_t)2 * (n_ranks + 1) * c->slot_bytes + (size_t)(2 * n_ranks + 2) * c->fc * 4;
    cudaError_t e = cudaMalloc(&c->d_buf, c->buf_bytes);
    if (e == cudaSuccess) e = cudaMemset(c->d_buf, 0, c->buf_bytes);
    if (e == cudaSuccess) e = cudaMalloc(&c->d_peers, sizeof(char*) * 8);
    if (e == cudaSuccess) e = cudaMalloc(&c->d_state, sizeof(unsigned int) * 2);
    if (e == cudaSuccess) e = cudaMemset(c->d_state, 0, sizeof(unsigned int) * 2);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        free_comm(c);
        delete c;
        cudaGetLastError();
        throw Error(G4Q_ERR_MEMORY_GUARD, std::string("communicator allocation failed: ") + cudaGetErrorString(e));
    }
    c->peer[rank] = c->d_buf;
    if (n_ranks == 1) {
        check_cuda(cudaMemcpy(c->d_peers, c->peer, sizeof(char*) * 8, cudaMemcpyHostToDevice), "communicator peers");
        c->peers_set = true;
    }
    c->magic = kCommMagic;
    return c;
}

void comm_buffer(const void* h, void** buf, uint64_t* bytes) {
    const Comm* c = checked_comm(h);
    if (buf) *buf = c->d_buf;
    if (bytes) *bytes = c->buf_bytes;
}

void comm_set_peers(void* h, void* const* peer_bufs) {
    Comm* c = checked_comm(h);
    if (!peer_bufs) throw Error(G4Q_ERR_INVALID_ARGUMENT, "peer buffer array must be non-null");
    for (int r = 0; r < c->n_ranks; ++r) {
        if (r == c->rank) continue;
        if (!peer_bufs[r]) throw Error(G4Q_ERR_INVALID_ARGUMENT, "missing exchange buffer of rank " + std::to_string(r));
        c->peer[r] = static_cast<char*>(peer_bufs[r]);
    }
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(c->device);
    const cudaError_t e = cudaMemcpy(c->d_peers, c->peer, sizeof(char*) * 8, cudaMemcpyHostToDevice);
    cudaSetDevice(prev);
    check_cuda(e, "communicator peers");
    c->peers_set = true;
}

void comm_allreduce(void* h, void* data, int64_t count, int dtype, cudaStream_t st) {
    Comm* c = checked_comm(h);
    if (c->device != current_device()) throw Error(G4Q_ERR_INVALID_ARGUMENT, "communicator belongs to another device");
    if (dtype != G4Q_DTYPE_BF16 && dtype != G4Q_DTYPE_F32)
        throw Error(G4Q_ERR_INVALID_ARGUMENT, "dtype must be G4Q_DTYPE_BF16 or G4Q_DTYPE_F32");
    const int esize = dtype == G4Q_DTYPE_BF16 ? 2 : 4;
    if (count < 0 || count > c->max_elems)
        throw Error(G4Q_ERR_INVALID_ARGUMENT, "count must be in [0, " + std::to_string(c->max_elems) + "]");
    if (count == 0 || c->n_ranks == 1) return;
    if (!data || (reinterpret_cast<uintptr_t>(data) & 15u) != 0 || (count * esize) % 16 != 0)
        throw Error(G4Q_ERR_INVALID_ARGUMENT, "data must be 16-byte aligned and count * element size a multiple of 16");
    if (!c->peers_set) throw Error(G4Q_ERR_INVALID_ARGUMENT, "communicator peers not set");
    ArArgs a{};
    a.data = data;
    a.count = count;
    a.esize = esize;
    a.rank = c->rank;
    a.n_ranks = c->n_ranks;
    a.two_shot = count * esize > kOneShotBytes ? 1 : 0;
    a.slot_bytes = c->slot_bytes;
    a.fc = c->fc;
    a.peers = c->d_peers;
    a.state = c->d_state;
    a.err = device_scratch().err;
    const int64_t nch = (count + kChunk - 1) / kChunk;
    const int grid = (int)(nch < device_sm_count() ? nch : device_sm_count());
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kCommThreads);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;   // CTAs wait on each other's chunks across ranks
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    check_cuda(cudaLaunchKernelEx(&cfg, allreduce_kernel, a), "allreduce launch");
}

void comm_free(void* h) {
    Comm* c = checked_comm(h);
    c->magic = 0;
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(c->device);
    free_comm(c);
    cudaSetDevice(prev);
    delete c;
}

}  // namespace g4q
