// g4q_api.cu -- the extern "C" boundary of libg4q (include/g4q.h).
//
// Mirrors the reference's C ABI conventions (native/gemma4_mlx/src/runtime.cc): a status
// code per call, a thread-local last-error buffer (runtime.cc:46, 115-133, 816-823),
// magic-tagged opaque handles allocated with new(std::nothrow) and invalidated on free
// (runtime.cc:41-45, 841-846, 900-912), and no C++ exception crossing the boundary.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <new>
#include <string>

#include "g4q.h"
#include "g4q_internal.h"

namespace g4q {

static thread_local char g_last_error[512] = "";

static G4qStatus fail(G4qStatus s, const std::string& msg) {
    std::snprintf(g_last_error, sizeof(g_last_error), "%s", msg.c_str());
    return s;
}

static G4qStatus ok() {
    g_last_error[0] = '\0';
    return G4Q_OK;
}

int current_device() {
    int d = 0;
    check_cuda(cudaGetDevice(&d), "cudaGetDevice");
    return d;
}

int device_sm_count() {
    static int cache[64] = {0};
    const int d = current_device();
    if (cache[d & 63] == 0) {
        int n = 0;
        check_cuda(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, d), "cudaDeviceGetAttribute");
        cache[d & 63] = n;
    }
    return cache[d & 63];
}

size_t max_dynamic_smem(const void* kernel) {
    int optin = 0;
    check_cuda(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, current_device()),
               "cudaDeviceGetAttribute(smem optin)");
    cudaFuncAttributes fa;
    check_cuda(cudaFuncGetAttributes(&fa, kernel), "cudaFuncGetAttributes");
    return (size_t)optin - fa.sharedSizeBytes;
}

static std::mutex g_scratch_mu;

static DeviceScratch g_per_dev[64];

DeviceScratch* device_scratch_if_created() {
    const int d = current_device();
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    DeviceScratch& s = g_per_dev[d & 63];
    return s.err != nullptr ? &s : nullptr;
}

DeviceScratch& device_scratch() {
    const int d = current_device();
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    DeviceScratch& s = g_per_dev[d & 63];
    if (s.err == nullptr) {
        constexpr int64_t kRows = 65536, kQuads = 65536;
        int* err = nullptr;
        float* rms = nullptr;
        int* counters = nullptr;
        check_cuda(cudaMalloc(&err, sizeof(int)), "cudaMalloc(device error word)");
        cudaError_t e = cudaMalloc(&rms, kRows * sizeof(float));
        if (e == cudaSuccess) e = cudaMalloc(&counters, kQuads * sizeof(int));
        if (e == cudaSuccess) e = cudaMemset(err, 0, sizeof(int));
        if (e == cudaSuccess) e = cudaMemset(counters, 0, kQuads * sizeof(int));
        if (e == cudaSuccess) e = cudaDeviceSynchronize();
        if (e != cudaSuccess) {
            cudaFree(err);
            cudaFree(rms);
            cudaFree(counters);
            check_cuda(e, "device scratch");
        }
        s.rms = rms;
        s.rms_rows = kRows;
        s.counters = counters;
        s.counters_n = kQuads;
        s.err = err;
    }
    return s;
}

void reserve_gemv_scratch(int64_t N, int64_t K) {
    DeviceScratch& s = device_scratch();
    const size_t need = gemv2_slots_bytes(N, K, device_sm_count());
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    if (need <= s.slots_bytes) return;
    // The old slots are never freed: a CUDA graph captured earlier with g4q_qmm has their address
    // baked into its kernel arguments and may still be replayed. They stay allocated until the
    // process exits (the sizes only grow, so the retired buffers add up to less than the new one).
    float* grown = nullptr;
    check_cuda(cudaMalloc(&grown, need), "cudaMalloc(gemv slots)");
    s.slots = grown;
    s.slots_bytes = need;
}

// Runs an entry point body, translating exceptions into a status + message.
template <typename F>
static G4qStatus guarded(const char* fn, F&& body) {
    try {
        body();
        return ok();
    } catch (const Error& e) {
        return fail(e.status, std::string(fn) + ": " + e.what());
    } catch (const std::bad_alloc&) {
        return fail(G4Q_ERR_MEMORY_GUARD, std::string(fn) + ": host allocation failed");
    } catch (const std::exception& e) {
        return fail(G4Q_ERR_RUNTIME, std::string(fn) + ": " + e.what());
    } catch (...) {
        return fail(G4Q_ERR_RUNTIME, std::string(fn) + ": unknown native error");
    }
}

static void require(bool cond, G4qStatus s, const std::string& msg) {
    if (!cond) throw Error(s, msg);
}

static Weight* checked(const G4qWeight* h, const char* what) {
    auto* w = reinterpret_cast<Weight*>(const_cast<G4qWeight*>(h));
    require(w != nullptr, G4Q_ERR_INVALID_ARGUMENT, std::string(what) + " requires a non-null weight handle");
    require(w->magic == kWeightMagic, G4Q_ERR_INVALID_ARGUMENT, std::string(what) + " received an invalid weight handle");
    require(w->device == current_device(), G4Q_ERR_INVALID_ARGUMENT,
            std::string(what) + ": the current CUDA device is not the handle's device");
    return w;
}

static bool device_accessible(const void* p) {
    cudaPointerAttributes attr;
    if (cudaPointerGetAttributes(&attr, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return attr.type == cudaMemoryTypeDevice || attr.type == cudaMemoryTypeManaged;
}

static void require_aligned16(const void* p, const char* what) {
    require((reinterpret_cast<uintptr_t>(p) & 15u) == 0, G4Q_ERR_INVALID_ARGUMENT,
            std::string(what) + " must be 16-byte aligned");
}

}  // namespace g4q

using namespace g4q;

extern "C" {

G4qStatus g4q_runtime_version(G4qVersionInfo* out) {
    if (out == nullptr) return fail(G4Q_ERR_INVALID_ARGUMENT, "g4q_runtime_version requires a non-null out pointer");
    out->abi_version = G4Q_ABI_VERSION;
    out->backend_name = "g4q_b200";
    out->backend_version = "sm_100a tcgen05/mma-sync affine-q4g64 v1";
    return ok();
}

G4qStatus g4q_get_last_error(char* buffer, size_t buffer_len) {
    if (buffer == nullptr || buffer_len == 0)
        return fail(G4Q_ERR_INVALID_ARGUMENT, "g4q_get_last_error requires a writable buffer");
    std::snprintf(buffer, buffer_len, "%s", g_last_error);
    return G4Q_OK;
}

G4qStatus g4q_weight_create(int64_t rows, int64_t cols, int32_t bits, int32_t group_size, G4qWeight** out) {
    return guarded("g4q_weight_create", [&] {
        require(out != nullptr, G4Q_ERR_INVALID_ARGUMENT, "requires a non-null out pointer");
        *out = nullptr;
        require(rows > 0 && cols > 0, G4Q_ERR_INVALID_ARGUMENT, "rows and cols must be positive");
        require((bits == 4 || bits == 8) && (group_size == 32 || group_size == 64 || group_size == 128),
                G4Q_ERR_UNSUPPORTED_CONFIG,
                "supported quantization: bits 4 or 8, group_size 32, 64 or 128 (got bits=" + std::to_string(bits) +
                    ", group_size=" + std::to_string(group_size) + ")");
        if (bits != 4 || group_size != 64) {
            // other specs of the manifest stay in MLX's layout and run on the generic kernels
            require(cols % group_size == 0, G4Q_ERR_UNSUPPORTED_CONFIG, "cols must be a multiple of group_size");
            (void)device_scratch();
            Weight* w = new (std::nothrow) Weight();
            require(w != nullptr, G4Q_ERR_MEMORY_GUARD, "host allocation failed");
            w->N = rows;
            w->K = cols;
            w->bits = bits;
            w->group_size = group_size;
            w->device = current_device();
            w->mlx = true;
            w->small_scales = false;
            const size_t pb = (size_t)rows * cols * bits / 8, gb = (size_t)rows * (cols / group_size) * 2;
            cudaError_t e = cudaMalloc(&w->packed, pb);
            if (e == cudaSuccess) e = cudaMalloc(&w->mlx_scales, gb);
            if (e == cudaSuccess) e = cudaMalloc(&w->mlx_biases, gb);
            if (e == cudaSuccess) e = cudaMalloc(&w->d_flags, sizeof(int));
            if (e == cudaSuccess) e = cudaMemset(w->d_flags, 0, sizeof(int));
            if (e != cudaSuccess) {
                cudaFree(w->packed);
                cudaFree(w->mlx_scales);
                cudaFree(w->mlx_biases);
                cudaFree(w->d_flags);
                delete w;
                cudaGetLastError();
                throw Error(G4Q_ERR_MEMORY_GUARD, std::string("device allocation failed: ") + cudaGetErrorString(e));
            }
            w->bytes = pb + 2 * gb;
            w->magic = kWeightMagic;
            *out = reinterpret_cast<G4qWeight*>(w);
            return;
        }
        require(rows % 16 == 0, G4Q_ERR_UNSUPPORTED_CONFIG, "rows must be a multiple of 16");
        require(cols % 64 == 0, G4Q_ERR_UNSUPPORTED_CONFIG, "cols must be a multiple of 64");
        (void)device_scratch();   // per-device library state exists before any compute call
        require(rows / 64 <= device_scratch().counters_n, G4Q_ERR_UNSUPPORTED_CONFIG, "rows exceed 4,194,304");
        reserve_gemv_scratch(rows, cols);
        Weight* w = new (std::nothrow) Weight();
        require(w != nullptr, G4Q_ERR_MEMORY_GUARD, "host allocation failed");
        w->N = rows;
        w->K = cols;
        w->bits = bits;
        w->group_size = group_size;
        w->device = current_device();
        const size_t packed_bytes = (size_t)rows * cols / 2, sb_bytes = (size_t)rows * (cols / 64) * 4;
        cudaError_t e = cudaMalloc(&w->packed, packed_bytes);
        if (e == cudaSuccess) e = cudaMalloc(&w->sb, sb_bytes);
        if (e == cudaSuccess) e = cudaMalloc(&w->d_flags, sizeof(int));
        if (e == cudaSuccess) e = cudaMalloc(&w->argmax_scratch, 17 * sizeof(unsigned long long));
        if (e == cudaSuccess) e = cudaMemset(w->d_flags, 0, sizeof(int));
        if (e == cudaSuccess) e = cudaMemset(w->argmax_scratch, 0, 17 * sizeof(unsigned long long));
        if (e != cudaSuccess) {
            cudaFree(w->packed);
            cudaFree(w->sb);
            cudaFree(w->d_flags);
            cudaFree(w->argmax_scratch);
            delete w;
            cudaGetLastError();
            throw Error(G4Q_ERR_MEMORY_GUARD, std::string("device allocation failed: ") + cudaGetErrorString(e));
        }
        w->bytes = packed_bytes + sb_bytes;
        w->magic = kWeightMagic;
        *out = reinterpret_cast<G4qWeight*>(w);
    });
}

G4qStatus g4q_weight_free(G4qWeight* h) {
    return guarded("g4q_weight_free", [&] {
        auto* w = reinterpret_cast<Weight*>(h);
        require(w != nullptr, G4Q_ERR_INVALID_ARGUMENT, "requires a non-null weight handle");
        require(w->magic == kWeightMagic, G4Q_ERR_INVALID_ARGUMENT, "received an invalid weight handle");
        w->magic = 0;
        int prev = 0;
        cudaGetDevice(&prev);
        cudaSetDevice(w->device);
        cudaFree(w->packed);
        cudaFree(w->sb);
        cudaFree(w->d_flags);
        cudaFree(w->argmax_scratch);
        cudaFree(w->mlx_scales);
        cudaFree(w->mlx_biases);
        cudaSetDevice(prev);
        delete w;
    });
}

// Repacked-weight cache file: header, then packed words, then scale|bias words.
struct CacheHeader {
    char magic[8];            // "G4QWCACH"
    uint32_t version;         // 1
    uint32_t layout;          // 1: kernel layout v1
    int64_t rows, cols;
    int32_t bits, group_size;
    uint64_t packed_bytes, sb_bytes;
    uint64_t checksum;        // FNV-1a 64 over the payload
};
static_assert(sizeof(CacheHeader) == 64, "cache header is 64 bytes");
static const char kCacheMagic[8] = {'G', '4', 'Q', 'W', 'C', 'A', 'C', 'H'};

static uint64_t fnv1a(const unsigned char* p, size_t n, uint64_t h = 0xcbf29ce484222325ull) {
    for (size_t i = 0; i < n; ++i) h = (h ^ p[i]) * 0x100000001b3ull;
    return h;
}

G4qStatus g4q_weight_save(const G4qWeight* h, const char* path) {
    return guarded("g4q_weight_save", [&] {
        Weight* w = checked(h, "g4q_weight_save");
        require(path != nullptr, G4Q_ERR_INVALID_ARGUMENT, "path must be non-null");
        require(!w->mlx, G4Q_ERR_UNSUPPORTED_CONFIG, "the cache holds 4-bit group-64 handles only");
        CacheHeader hd{};
        std::memcpy(hd.magic, kCacheMagic, 8);
        hd.version = 1;
        hd.layout = 1;
        hd.rows = w->N;
        hd.cols = w->K;
        hd.bits = 4;
        hd.group_size = 64;
        hd.packed_bytes = (uint64_t)w->N * w->K / 2;
        hd.sb_bytes = (uint64_t)w->N * (w->K / 64) * 4;
        std::string buf(hd.packed_bytes + hd.sb_bytes, '\0');
        check_cuda(cudaMemcpy(&buf[0], w->packed, hd.packed_bytes, cudaMemcpyDeviceToHost), "read packed words");
        check_cuda(cudaMemcpy(&buf[hd.packed_bytes], w->sb, hd.sb_bytes, cudaMemcpyDeviceToHost), "read scale words");
        hd.checksum = fnv1a(reinterpret_cast<const unsigned char*>(buf.data()), buf.size());
        FILE* f = std::fopen(path, "wb");
        require(f != nullptr, G4Q_ERR_RUNTIME, std::string("cannot open ") + path + " for writing");
        const bool okw = std::fwrite(&hd, sizeof(hd), 1, f) == 1 && std::fwrite(buf.data(), 1, buf.size(), f) == buf.size();
        const bool okc = std::fclose(f) == 0;
        require(okw && okc, G4Q_ERR_RUNTIME, std::string("writing ") + path + " failed");
    });
}

G4qStatus g4q_weight_open(const char* path, G4qWeight** out) {
    return guarded("g4q_weight_open", [&] {
        require(out != nullptr && path != nullptr, G4Q_ERR_INVALID_ARGUMENT, "path and out must be non-null");
        *out = nullptr;
        FILE* f = std::fopen(path, "rb");
        require(f != nullptr, G4Q_ERR_MODEL_LOAD, std::string("cannot open ") + path);
        CacheHeader hd{};
        const bool got = std::fread(&hd, sizeof(hd), 1, f) == 1;
        std::string buf;
        bool ok_hdr = got && std::memcmp(hd.magic, kCacheMagic, 8) == 0 && hd.version == 1 && hd.layout == 1 &&
                      hd.bits == 4 && hd.group_size == 64 && hd.rows > 0 && hd.cols > 0 && hd.rows % 16 == 0 &&
                      hd.cols % 64 == 0 && hd.rows <= (int64_t)1 << 31 && hd.cols <= (int64_t)1 << 31 &&
                      hd.packed_bytes == (uint64_t)hd.rows * hd.cols / 2 &&
                      hd.sb_bytes == (uint64_t)hd.rows * (hd.cols / 64) * 4;
        bool ok_payload = false;
        if (ok_hdr) {
            buf.resize(hd.packed_bytes + hd.sb_bytes);
            ok_payload = std::fread(&buf[0], 1, buf.size(), f) == buf.size() && std::fgetc(f) == EOF &&
                         fnv1a(reinterpret_cast<const unsigned char*>(buf.data()), buf.size()) == hd.checksum;
        }
        std::fclose(f);
        require(ok_hdr, G4Q_ERR_MODEL_LOAD, std::string(path) + " is not a version-1 g4q weight cache file");
        require(ok_payload, G4Q_ERR_MODEL_LOAD, std::string(path) + ": payload size or checksum mismatch");
        G4qWeight* hw = nullptr;
        const G4qStatus st = g4q_weight_create(hd.rows, hd.cols, 4, 64, &hw);
        if (st != G4Q_OK) throw Error(st, "creating the handle failed");
        Weight* w = reinterpret_cast<Weight*>(hw);
        cudaError_t e = cudaMemcpy(w->packed, buf.data(), hd.packed_bytes, cudaMemcpyHostToDevice);
        if (e == cudaSuccess) e = cudaMemcpy(w->sb, buf.data() + hd.packed_bytes, hd.sb_bytes, cudaMemcpyHostToDevice);
        int flags = 0;
        if (e == cudaSuccess) {
            try {
                launch_sb_flags(*w, nullptr);
            } catch (...) {
                e = cudaErrorLaunchFailure;
            }
        }
        if (e == cudaSuccess) e = cudaMemcpy(&flags, w->d_flags, sizeof(int), cudaMemcpyDeviceToHost);
        if (e != cudaSuccess) {
            g4q_weight_free(hw);
            check_cuda(e, "uploading the cached buffers");
        }
        w->fast_ok = (flags & 1) == 0;
        w->small_scales = (flags & 4) == 0;
        w->subnormal_scales = (flags & 8) != 0;
        *out = hw;
    });
}

G4qStatus g4q_weight_info(const G4qWeight* h, G4qWeightInfo* out) {
    return guarded("g4q_weight_info", [&] {
        Weight* w = checked(h, "g4q_weight_info");
        require(out != nullptr, G4Q_ERR_INVALID_ARGUMENT, "requires a non-null out pointer");
        int flags = 0;
        check_cuda(cudaMemcpy(&flags, w->d_flags, sizeof(int), cudaMemcpyDeviceToHost), "read handle flags");
        out->rows = w->N;
        out->cols = w->K;
        out->bits = w->bits;
        out->group_size = w->group_size;
        out->device_bytes = w->bytes;
        out->device = w->device;
        out->fast_path_ok = (flags & 1) ? 0 : 1;
        out->error_flags = flags & 2;
    });
}

G4qStatus g4q_weight_load(G4qWeight* h, int64_t dst_row0, const uint32_t* packed, const uint16_t* scales,
                          const uint16_t* biases, int64_t src_rows, int64_t src_cols, int64_t src_row0,
                          int64_t src_k0, int64_t n_rows, void* stream) {
    return guarded("g4q_weight_load", [&] {
        Weight* w = checked(h, "g4q_weight_load");
        require(packed && scales && biases, G4Q_ERR_INVALID_ARGUMENT, "packed, scales and biases must be non-null");
        if (w->mlx) {   // MLX layout: copy the row / column window as it is (host or device source)
            const int64_t gs = w->group_size, per = 32 / w->bits;
            require(src_rows > 0 && src_cols > 0 && src_cols % gs == 0, G4Q_ERR_INVALID_ARGUMENT,
                    "source shape must be positive with cols a multiple of group_size");
            require(src_k0 >= 0 && src_k0 % gs == 0 && src_k0 + w->K <= src_cols, G4Q_ERR_INVALID_ARGUMENT,
                    "column window must be group aligned and inside the source");
            require(n_rows > 0 && src_row0 >= 0 && src_row0 + n_rows <= src_rows, G4Q_ERR_INVALID_ARGUMENT,
                    "row window must be inside the source");
            require(dst_row0 >= 0 && dst_row0 + n_rows <= w->N, G4Q_ERR_INVALID_ARGUMENT,
                    "destination rows must be inside the handle");
            cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
            const int64_t src_w = src_cols / per, dst_w = w->K / per, src_g = src_cols / gs, dst_g = w->K / gs;
            check_cuda(cudaMemcpy2DAsync(w->packed + dst_row0 * dst_w, dst_w * 4, packed + src_row0 * src_w + src_k0 / per,
                                         src_w * 4, dst_w * 4, n_rows, cudaMemcpyDefault, st),
                       "copy packed words");
            check_cuda(cudaMemcpy2DAsync(w->mlx_scales + dst_row0 * dst_g, dst_g * 2, scales + src_row0 * src_g + src_k0 / gs,
                                         src_g * 2, dst_g * 2, n_rows, cudaMemcpyDefault, st),
                       "copy scales");
            check_cuda(cudaMemcpy2DAsync(w->mlx_biases + dst_row0 * dst_g, dst_g * 2, biases + src_row0 * src_g + src_k0 / gs,
                                         src_g * 2, dst_g * 2, n_rows, cudaMemcpyDefault, st),
                       "copy biases");
            check_cuda(cudaStreamSynchronize(st), "weight copy");
            return;
        }
        require(src_rows > 0 && src_cols > 0 && src_cols % 64 == 0, G4Q_ERR_INVALID_ARGUMENT,
                "source shape must be positive with cols % 64 == 0");
        require(src_k0 >= 0 && src_k0 % 64 == 0 && src_k0 + w->K <= src_cols, G4Q_ERR_INVALID_ARGUMENT,
                "column window must be group aligned and inside the source");
        require(n_rows > 0 && n_rows % 16 == 0 && src_row0 >= 0 && src_row0 + n_rows <= src_rows,
                G4Q_ERR_INVALID_ARGUMENT, "row window must be a positive multiple of 16 inside the source");
        require(dst_row0 >= 0 && dst_row0 % 16 == 0 && dst_row0 + n_rows <= w->N, G4Q_ERR_INVALID_ARGUMENT,
                "destination rows must be 16-aligned and inside the handle");
        cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
        const int64_t ld_words = src_cols / 8, ld_groups = src_cols / 64;
        const bool on_device = device_accessible(packed) && device_accessible(scales) && device_accessible(biases);
        if (on_device) {
            launch_repack(packed, scales, biases, ld_words, ld_groups, src_row0, src_k0, n_rows, *w, dst_row0, st);
        } else {
            // host source: stage the row window on the device, then repack
            uint32_t* dw = nullptr;
            uint16_t *ds = nullptr, *db = nullptr;
            const size_t wb = (size_t)n_rows * ld_words * 4, gb = (size_t)n_rows * ld_groups * 2;
            cudaError_t e = cudaMalloc(&dw, wb);
            if (e == cudaSuccess) e = cudaMalloc(&ds, gb);
            if (e == cudaSuccess) e = cudaMalloc(&db, gb);
            if (e == cudaSuccess)
                e = cudaMemcpyAsync(dw, packed + src_row0 * ld_words, wb, cudaMemcpyHostToDevice, st);
            if (e == cudaSuccess)
                e = cudaMemcpyAsync(ds, scales + src_row0 * ld_groups, gb, cudaMemcpyHostToDevice, st);
            if (e == cudaSuccess)
                e = cudaMemcpyAsync(db, biases + src_row0 * ld_groups, gb, cudaMemcpyHostToDevice, st);
            if (e == cudaSuccess) {
                try {
                    launch_repack(dw, ds, db, ld_words, ld_groups, 0, src_k0, n_rows, *w, dst_row0, st);
                } catch (...) {
                    e = cudaErrorLaunchFailure;
                }
            }
            if (e == cudaSuccess) e = cudaStreamSynchronize(st);
            cudaFree(dw);
            cudaFree(ds);
            cudaFree(db);
            check_cuda(e, "staging a host-memory source");
        }
        check_cuda(cudaStreamSynchronize(st), "repack");
        int flags = 0;
        check_cuda(cudaMemcpy(&flags, w->d_flags, sizeof(int), cudaMemcpyDeviceToHost), "read handle flags");
        w->fast_ok = (flags & 1) == 0;   // cached so compute calls never read device memory
        w->small_scales = (flags & 4) == 0;
        w->subnormal_scales = (flags & 8) != 0;
    });
}

G4qStatus g4q_weight_export(const G4qWeight* h, uint32_t* packed, uint16_t* scales, uint16_t* biases,
                            void* stream) {
    return guarded("g4q_weight_export", [&] {
        Weight* w = checked(h, "g4q_weight_export");
        require(packed && scales && biases, G4Q_ERR_INVALID_ARGUMENT, "outputs must be non-null device pointers");
        if (w->mlx) {
            cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
            const size_t pb = (size_t)w->N * w->K * w->bits / 8, gb = (size_t)w->N * (w->K / w->group_size) * 2;
            check_cuda(cudaMemcpyAsync(packed, w->packed, pb, cudaMemcpyDefault, st), "export packed words");
            check_cuda(cudaMemcpyAsync(scales, w->mlx_scales, gb, cudaMemcpyDefault, st), "export scales");
            check_cuda(cudaMemcpyAsync(biases, w->mlx_biases, gb, cudaMemcpyDefault, st), "export biases");
            return;
        }
        launch_export(*w, packed, scales, biases, reinterpret_cast<cudaStream_t>(stream));
    });
}

G4qStatus g4q_dequantize(const G4qWeight* h, const int32_t* row_ids, int64_t n_ids, uint16_t* out, int32_t chain,
                         void* stream) {
    return guarded("g4q_dequantize", [&] {
        Weight* w = checked(h, "g4q_dequantize");
        require(out != nullptr, G4Q_ERR_INVALID_ARGUMENT, "out must be non-null");
        require(chain == G4Q_CHAIN_R1 || chain == G4Q_CHAIN_R2, G4Q_ERR_INVALID_ARGUMENT, "chain must be 1 (R1) or 2 (R2)");
        require(row_ids == nullptr || n_ids >= 0, G4Q_ERR_INVALID_ARGUMENT, "n_ids must be >= 0");
        require_aligned16(out, "out");
        if (w->mlx) {
            cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
            if (row_ids == nullptr)
                launch_dequantize_mlx(w->packed, w->mlx_scales, w->mlx_biases, w->N, w->K, w->bits, w->group_size,
                                      chain, out, st);
            else
                launch_dequantize_mlx_rows(*w, row_ids, n_ids, out, chain, st);
            return;
        }
        launch_dequantize(*w, row_ids, n_ids, out, chain, w->d_flags, reinterpret_cast<cudaStream_t>(stream));
    });
}

G4qStatus g4q_dequantize_mlx(const uint32_t* packed, const uint16_t* scales, const uint16_t* biases, int64_t rows,
                             int64_t cols, int32_t bits, int32_t group_size, int32_t chain, uint16_t* out,
                             void* stream) {
    return guarded("g4q_dequantize_mlx", [&] {
        require(packed && scales && biases && out, G4Q_ERR_INVALID_ARGUMENT, "pointers must be non-null");
        require(bits == 4 || bits == 8, G4Q_ERR_UNSUPPORTED_CONFIG, "bits must be 4 or 8");
        require(group_size == 32 || group_size == 64 || group_size == 128, G4Q_ERR_UNSUPPORTED_CONFIG,
                "group_size must be 32, 64 or 128");
        require(rows >= 0 && cols > 0 && cols % group_size == 0, G4Q_ERR_INVALID_ARGUMENT,
                "cols must be a positive multiple of group_size");
        require(chain == G4Q_CHAIN_R1 || chain == G4Q_CHAIN_R2, G4Q_ERR_INVALID_ARGUMENT, "chain must be 1 (R1) or 2 (R2)");
        require((reinterpret_cast<uintptr_t>(out) & 3u) == 0, G4Q_ERR_INVALID_ARGUMENT, "out must be 4-byte aligned");
        if (rows == 0) return;
        launch_dequantize_mlx(packed, scales, biases, rows, cols, bits, group_size, chain, out,
                              reinterpret_cast<cudaStream_t>(stream));
    });
}

static void qmm_common(const char* fn, const G4qWeight* h, const uint16_t* x, int64_t M, int64_t ldx, void* y,
                       int64_t ldy, uint32_t flags, float eps, void* stream) {
    Weight* w = checked(h, fn);
    require(M >= 0, G4Q_ERR_INVALID_ARGUMENT, "M must be >= 0");
    if (M == 0) return;
    require(x != nullptr && y != nullptr, G4Q_ERR_INVALID_ARGUMENT, "x and y must be non-null");
    require((flags & ~(G4Q_QMM_RMS_SCALE | G4Q_QMM_OUT_F32)) == 0, G4Q_ERR_INVALID_ARGUMENT, "unknown flag bits");
    require(ldx >= w->K && ldx % 8 == 0, G4Q_ERR_INVALID_ARGUMENT, "ldx must be >= cols and a multiple of 8");
    require(ldy >= w->N, G4Q_ERR_INVALID_ARGUMENT, "ldy must be >= rows");
    require_aligned16(x, "x");
    QmmCall c{w, x, M, ldx, y, ldy, flags, eps};
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (w->mlx) {   // 8-bit or non-64 groups: the generic kernel
        launch_qmm_mlx(c, st);
        return;
    }
    require(w->fast_ok, G4Q_ERR_UNSUPPORTED_CONFIG,
            "a scale is non-finite or |scale| >= 2^120; use g4q_dequantize for such weights");
    if (M <= 16)
        launch_gemv(c, st);
    else
        launch_gemm(c, st);
}

G4qStatus g4q_qmm(const G4qWeight* h, const uint16_t* x, int64_t M, int64_t ldx, uint16_t* y, int64_t ldy,
                  void* stream) {
    return guarded("g4q_qmm", [&] { qmm_common("g4q_qmm", h, x, M, ldx, y, ldy, 0u, 1e-6f, stream); });
}

G4qStatus g4q_qmm_ex(const G4qWeight* h, const uint16_t* x, int64_t M, int64_t ldx, void* y, int64_t ldy,
                     uint32_t flags, float eps, void* stream) {
    return guarded("g4q_qmm_ex", [&] { qmm_common("g4q_qmm_ex", h, x, M, ldx, y, ldy, flags, eps, stream); });
}

G4qStatus g4q_qmm_path(const G4qWeight* h, int64_t M, int32_t* kernel, int32_t* splits) {
    return guarded("g4q_qmm_path", [&] {
        Weight* w = checked(h, "g4q_qmm_path");
        require(M >= 1, G4Q_ERR_INVALID_ARGUMENT, "M must be >= 1");
        require(kernel != nullptr && splits != nullptr, G4Q_ERR_INVALID_ARGUMENT, "kernel and splits must be non-null");
        *splits = 0;
        if (w->mlx) {
            *kernel = G4Q_PATH_GENERIC;
            return;
        }
        QmmCall c{w, nullptr, M, w->K, nullptr, w->N, 0u, 1e-6f};
        if (M <= 16) {
            *kernel = gemv2_supported(c) ? G4Q_PATH_GEMV_STREAMK : G4Q_PATH_GEMV_CLUSTER;
            return;
        }
        *kernel = G4Q_PATH_GEMM;
        *splits = gemm_splits(M, w->N, w->K);
    });
}

G4qStatus g4q_qmm_norm(const G4qWeight* h, const uint16_t* x, int64_t M, int64_t ldx, const uint16_t* weight,
                       float eps, uint16_t* xn, int64_t ldxn, uint16_t* y, int64_t ldy, void* stream) {
    return guarded("g4q_qmm_norm", [&] {
        Weight* w = checked(h, "g4q_qmm_norm");
        require(M >= 0, G4Q_ERR_INVALID_ARGUMENT, "M must be >= 0");
        if (M == 0) return;
        require(x != nullptr && y != nullptr && weight != nullptr, G4Q_ERR_INVALID_ARGUMENT,
                "x, weight and y must be non-null");
        require(ldx >= w->K && ldx % 8 == 0, G4Q_ERR_INVALID_ARGUMENT, "ldx must be >= cols and a multiple of 8");
        require(ldy >= w->N, G4Q_ERR_INVALID_ARGUMENT, "ldy must be >= rows");
        require(w->K % 8 == 0, G4Q_ERR_UNSUPPORTED_CONFIG, "cols must be a multiple of 8");
        require(eps >= 0.0f && std::isfinite(eps), G4Q_ERR_INVALID_ARGUMENT, "eps must be finite and >= 0");
        require_aligned16(x, "x");
        require_aligned16(weight, "weight");
        if (xn != nullptr) {
            require(ldxn >= w->K && ldxn % 8 == 0, G4Q_ERR_INVALID_ARGUMENT, "ldxn must be >= cols and a multiple of 8");
            require_aligned16(xn, "xn");
        }
        cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
        QmmCall c{w, x, M, ldx, y, ldy, 0u, eps};
        c.norm_w = weight;
        c.xn = xn;
        c.ldxn = ldxn;
        if (!w->mlx && w->fast_ok && M <= 8 && gemv2_supported(c)) {
            launch_gemv2(c, st);   // the norm fused into the GEMV's x staging
            return;
        }
        require(xn != nullptr, G4Q_ERR_INVALID_ARGUMENT,
                "xn is required unless M <= 8 on a 4-bit group-64 weight the fused GEMV takes");
        launch_rms_norm(x, ldx, weight, M, w->K, eps, xn, ldxn, st);
        qmm_common("g4q_qmm_norm", h, xn, M, ldxn, y, ldy, 0u, eps, stream);
    });
}

G4qStatus g4q_qmm_geglu(const G4qWeight* h, const uint16_t* x, int64_t M, int64_t ldx, const uint16_t* norm_weight,
                        uint32_t flags, float eps, uint16_t* y, uint16_t* act, int64_t ld_act, void* stream) {
    return guarded("g4q_qmm_geglu", [&] {
        Weight* w = checked(h, "g4q_qmm_geglu");
        require(!w->mlx, G4Q_ERR_UNSUPPORTED_CONFIG, "the fused GeGLU takes a 4-bit group-64 weight");
        require(w->N % 64 == 0, G4Q_ERR_INVALID_ARGUMENT, "a paired gate|up weight has rows in multiples of 64");
        require(M >= 0, G4Q_ERR_INVALID_ARGUMENT, "M must be >= 0");
        if (M == 0) return;
        require(x != nullptr && act != nullptr, G4Q_ERR_INVALID_ARGUMENT, "x and act must be non-null");
        require((flags & ~G4Q_QMM_RMS_SCALE) == 0, G4Q_ERR_INVALID_ARGUMENT, "only G4Q_QMM_RMS_SCALE is accepted");
        require(ldx >= w->K && ldx % 8 == 0, G4Q_ERR_INVALID_ARGUMENT, "ldx must be >= cols and a multiple of 8");
        require(ld_act >= w->N / 2 && ld_act % 8 == 0, G4Q_ERR_INVALID_ARGUMENT,
                "ld_act must be >= rows/2 and a multiple of 8");
        require_aligned16(x, "x");
        require_aligned16(act, "act");
        require(w->fast_ok, G4Q_ERR_UNSUPPORTED_CONFIG, "a scale is non-finite or |scale| >= 2^120");
        cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
        QmmCall c{w, x, M, ldx, act, ld_act, flags, eps};
        c.geglu = true;
        if (norm_weight != nullptr) {
            require(flags == 0, G4Q_ERR_INVALID_ARGUMENT, "a norm weight and G4Q_QMM_RMS_SCALE exclude each other");
            require(eps >= 0.0f && std::isfinite(eps), G4Q_ERR_INVALID_ARGUMENT, "eps must be finite and >= 0");
            require(w->K % 8 == 0, G4Q_ERR_UNSUPPORTED_CONFIG, "cols must be a multiple of 8");
            require_aligned16(norm_weight, "norm_weight");
            c.norm_w = norm_weight;
        }
        if (M <= 8 && gemv2_supported(c)) {
            launch_gemv2(c, st);   // the GeGLU in the GEMV's epilogue (and the norm in its staging)
            return;
        }
        require(norm_weight == nullptr, G4Q_ERR_INVALID_ARGUMENT,
                "a norm weight is taken only where the fused GEMV runs (M <= 8); normalize with g4q_rms_norm first");
        if (M > 16) {
            launch_gemm(c, st);    // the GeGLU in the tcgen05 GEMM's epilogue (or its split-K reduction)
            return;
        }
        require(y != nullptr, G4Q_ERR_INVALID_ARGUMENT,
                "y is required for 9 <= M <= 16 and for M <= 8 on a shape the fused GEMV does not take");
        require_aligned16(y, "y");
        qmm_common("g4q_qmm_geglu", h, x, M, ldx, y, w->N, flags, eps, stream);
        // the pairs: per token, N/64 rows of 32 gate values followed by the 32 matching up values
        if (ld_act == w->N / 2) {
            launch_geglu(y, 64, y + 32, 64, act, 32, M * (w->N / 64), 32, st);
        } else {
            for (int64_t m = 0; m < M; ++m)
                launch_geglu(y + m * w->N, 64, y + m * w->N + 32, 64, act + m * ld_act, 32, w->N / 64, 32, st);
        }
    });
}

G4qStatus g4q_lm_head_argmax(const G4qWeight* h, const uint16_t* x, int64_t M, int64_t ldx, float softcap,
                             uint32_t flags, float eps, int64_t row_offset, uint16_t* logits, int64_t ld_logits,
                             int32_t* tokens, float* values, uint64_t* keys, void* stream) {
    return guarded("g4q_lm_head_argmax", [&] {
        Weight* w = checked(h, "g4q_lm_head_argmax");
        require(!w->mlx, G4Q_ERR_UNSUPPORTED_CONFIG, "the fused LM head takes a 4-bit group-64 weight");
        require(M >= 1 && M <= 16, G4Q_ERR_INVALID_ARGUMENT, "M must be in [1, 16]");
        require(x != nullptr, G4Q_ERR_INVALID_ARGUMENT, "x must be non-null");
        require((flags & ~G4Q_QMM_RMS_SCALE) == 0, G4Q_ERR_INVALID_ARGUMENT, "only G4Q_QMM_RMS_SCALE is accepted");
        require(ldx >= w->K && ldx % 8 == 0, G4Q_ERR_INVALID_ARGUMENT, "ldx must be >= cols and a multiple of 8");
        require(logits == nullptr || ld_logits >= w->N, G4Q_ERR_INVALID_ARGUMENT, "ld_logits must be >= rows");
        require(row_offset >= 0 && row_offset + w->N <= 0xFFFFFFFFll, G4Q_ERR_INVALID_ARGUMENT,
                "row_offset + rows must fit in 32 bits");
        require_aligned16(x, "x");
        require(w->fast_ok, G4Q_ERR_UNSUPPORTED_CONFIG, "a scale is non-finite or |scale| >= 2^120");
        launch_lm_head(*w, x, M, ldx, softcap, flags, eps, row_offset, logits, ld_logits, tokens, values,
                       reinterpret_cast<unsigned long long*>(keys), reinterpret_cast<cudaStream_t>(stream));
    });
}

G4qStatus g4q_lm_head_argmax_noalloc(const uint32_t* packed, const uint32_t* sb, int64_t rows, int64_t cols,
                                     const uint16_t* x, int64_t M, int64_t ldx, float softcap, uint32_t flags,
                                     float eps, int64_t row_offset, uint16_t* logits, int64_t ld_logits,
                                     int32_t* tokens, float* values, uint64_t* keys, void* stream) {
    return guarded("g4q_lm_head_argmax_noalloc", [&] {
        require(packed && sb && x, G4Q_ERR_INVALID_ARGUMENT, "packed, sb and x must be non-null device pointers");
        require(rows > 0 && rows % 16 == 0 && cols > 0 && cols % 64 == 0, G4Q_ERR_INVALID_ARGUMENT,
                "rows must be a positive multiple of 16 and cols of 64");
        require(M >= 1 && M <= 16, G4Q_ERR_INVALID_ARGUMENT,
                "M must be in [1, 16] (the static scratch holds 16 keys); got " + std::to_string(M));
        require((flags & ~G4Q_QMM_RMS_SCALE) == 0, G4Q_ERR_INVALID_ARGUMENT, "only G4Q_QMM_RMS_SCALE is accepted");
        require(ldx >= cols && ldx % 8 == 0, G4Q_ERR_INVALID_ARGUMENT, "ldx must be >= cols and a multiple of 8");
        require(logits == nullptr || ld_logits >= rows, G4Q_ERR_INVALID_ARGUMENT, "ld_logits must be >= rows");
        require(row_offset >= 0 && row_offset + rows <= 0xFFFFFFFFll, G4Q_ERR_INVALID_ARGUMENT,
                "row_offset + rows must fit in 32 bits");
        require_aligned16(x, "x");
        require_aligned16(packed, "packed");
        launch_lm_head_noalloc(packed, sb, rows, cols, x, M, ldx, softcap, flags, eps, row_offset, logits, ld_logits,
                               tokens, values, reinterpret_cast<unsigned long long*>(keys),
                               reinterpret_cast<cudaStream_t>(stream));
    });
}

G4qStatus g4q_decode_plan_create(const G4qDecodePhase* phases, int32_t n_phases, int32_t max_tokens,
                                 G4qDecodePlan** out) {
    return guarded("g4q_decode_plan_create", [&] {
        require(out != nullptr, G4Q_ERR_INVALID_ARGUMENT, "requires a non-null out pointer");
        *out = nullptr;
        *out = reinterpret_cast<G4qDecodePlan*>(decode_plan_create(phases, n_phases, max_tokens, 0, 1));
    });
}

G4qStatus g4q_decode_plan_create_ex(const G4qDecodePhase* phases, const G4qPhasePrologue* prologues,
                                    int32_t n_phases, int32_t max_tokens, int32_t rank, int32_t n_ranks,
                                    G4qDecodePlan** out) {
    return guarded("g4q_decode_plan_create_ex", [&] {
        require(out != nullptr, G4Q_ERR_INVALID_ARGUMENT, "requires a non-null out pointer");
        *out = nullptr;
        *out = reinterpret_cast<G4qDecodePlan*>(
            decode_plan_create(phases, n_phases, max_tokens, rank, n_ranks, prologues));
    });
}

G4qStatus g4q_decode_plan_create_tp(const G4qDecodePhase* phases, int32_t n_phases, int32_t max_tokens,
                                    int32_t rank, int32_t n_ranks, G4qDecodePlan** out) {
    return guarded("g4q_decode_plan_create_tp", [&] {
        require(out != nullptr, G4Q_ERR_INVALID_ARGUMENT, "requires a non-null out pointer");
        *out = nullptr;
        *out = reinterpret_cast<G4qDecodePlan*>(decode_plan_create(phases, n_phases, max_tokens, rank, n_ranks));
    });
}

G4qStatus g4q_decode_plan_trace(G4qDecodePlan* plan, uint64_t* buffer, int64_t* words) {
    return guarded("g4q_decode_plan_trace", [&] {
        require(words != nullptr, G4Q_ERR_INVALID_ARGUMENT, "words must be non-null");
        const int64_t need = decode_plan_trace_words(plan);
        decode_plan_set_trace(plan, buffer, need);
        *words = need;
    });
}

G4qStatus g4q_decode_plan_buffers(G4qDecodePlan* plan, void** slots, uint64_t* slot_bytes, void** xkeys,
                                  uint64_t* xkey_bytes) {
    return guarded("g4q_decode_plan_buffers",
                   [&] { decode_plan_buffers(plan, slots, slot_bytes, xkeys, xkey_bytes); });
}

G4qStatus g4q_decode_plan_set_peers(G4qDecodePlan* plan, void* const* slots, void* const* xkeys) {
    return guarded("g4q_decode_plan_set_peers", [&] { decode_plan_set_peers(plan, slots, xkeys); });
}

G4qStatus g4q_comm_create(int32_t rank, int32_t n_ranks, int64_t max_elems, G4qComm** out) {
    return guarded("g4q_comm_create", [&] {
        require(out != nullptr, G4Q_ERR_INVALID_ARGUMENT, "requires a non-null out pointer");
        *out = nullptr;
        *out = reinterpret_cast<G4qComm*>(comm_create(rank, n_ranks, max_elems));
    });
}

G4qStatus g4q_comm_buffer(const G4qComm* comm, void** buffer, uint64_t* bytes) {
    return guarded("g4q_comm_buffer", [&] { comm_buffer(comm, buffer, bytes); });
}

G4qStatus g4q_comm_set_peers(G4qComm* comm, void* const* peer_buffers) {
    return guarded("g4q_comm_set_peers", [&] { comm_set_peers(comm, peer_buffers); });
}

G4qStatus g4q_allreduce(G4qComm* comm, void* data, int64_t count, int32_t dtype, void* stream) {
    return guarded("g4q_allreduce",
                   [&] { comm_allreduce(comm, data, count, dtype, reinterpret_cast<cudaStream_t>(stream)); });
}

G4qStatus g4q_comm_free(G4qComm* comm) {
    return guarded("g4q_comm_free", [&] { comm_free(comm); });
}

G4qStatus g4q_ipc_handle(const void* device_ptr, uint8_t* handle) {
    return guarded("g4q_ipc_handle", [&] {
        require(device_ptr != nullptr && handle != nullptr, G4Q_ERR_INVALID_ARGUMENT, "requires non-null pointers");
        cudaIpcMemHandle_t h;
        check_cuda(cudaIpcGetMemHandle(&h, const_cast<void*>(device_ptr)), "cudaIpcGetMemHandle");
        static_assert(sizeof(h) == G4Q_IPC_HANDLE_BYTES, "CUDA IPC handle size");
        memcpy(handle, &h, sizeof(h));
    });
}

G4qStatus g4q_ipc_open(const uint8_t* handle, void** device_ptr) {
    return guarded("g4q_ipc_open", [&] {
        require(device_ptr != nullptr && handle != nullptr, G4Q_ERR_INVALID_ARGUMENT, "requires non-null pointers");
        cudaIpcMemHandle_t h;
        memcpy(&h, handle, sizeof(h));
        *device_ptr = nullptr;
        check_cuda(cudaIpcOpenMemHandle(device_ptr, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
    });
}

G4qStatus g4q_ipc_close(void* device_ptr) {
    return guarded("g4q_ipc_close", [&] {
        require(device_ptr != nullptr, G4Q_ERR_INVALID_ARGUMENT, "requires a non-null pointer");
        check_cuda(cudaIpcCloseMemHandle(device_ptr), "cudaIpcCloseMemHandle");
    });
}

G4qStatus g4q_decode_plan_run(G4qDecodePlan* plan, int64_t M, float eps, float softcap, int64_t row_offset,
                              int32_t* tokens, float* values, uint64_t* keys, uint16_t* logits, int64_t ld_logits,
                              void* stream) {
    return guarded("g4q_decode_plan_run", [&] {
        require(row_offset >= 0 && row_offset < 0xFFFFFFFFll, G4Q_ERR_INVALID_ARGUMENT, "row_offset out of range");
        decode_plan_run(plan, (int)M, eps, softcap, row_offset, tokens, values, keys, logits, ld_logits,
                        reinterpret_cast<cudaStream_t>(stream));
    });
}

G4qStatus g4q_decode_plan_free(G4qDecodePlan* plan) {
    return guarded("g4q_decode_plan_free", [&] { decode_plan_free(plan); });
}

static Lora* checked_lora(const G4qLora* h, const char* what) {
    auto* l = reinterpret_cast<Lora*>(const_cast<G4qLora*>(h));
    require(l != nullptr, G4Q_ERR_INVALID_ARGUMENT, std::string(what) + " requires a non-null LoRA handle");
    require(l->magic == kLoraMagic, G4Q_ERR_INVALID_ARGUMENT, std::string(what) + " received an invalid LoRA handle");
    require(l->device == current_device(), G4Q_ERR_INVALID_ARGUMENT,
            std::string(what) + ": the current CUDA device is not the handle's device");
    return l;
}

// Round-to-nearest-even of a finite float to bf16, returned as a float (model_scalar's bf16 scalar).
static float round_to_bf16(float f) {
    uint32_t u;
    std::memcpy(&u, &f, sizeof(u));
    u = (u + 0x7FFFu + ((u >> 16) & 1u)) & 0xFFFF0000u;
    std::memcpy(&f, &u, sizeof(f));
    return f;
}

G4qStatus g4q_lora_create(int64_t rows, int64_t cols, int32_t rank, float alpha, const float* lora_a,
                          const float* lora_b, int32_t max_tokens, G4qLora** out) {
    return guarded("g4q_lora_create", [&] {
        require(out != nullptr, G4Q_ERR_INVALID_ARGUMENT, "out must be non-null");
        *out = nullptr;
        require(rank > 0, G4Q_ERR_INVALID_ARGUMENT, "LoRA rank must be greater than zero");
        require(alpha > 0.0f && std::isfinite(alpha), G4Q_ERR_INVALID_ARGUMENT, "LoRA alpha must be finite and positive");
        require(rank <= 256, G4Q_ERR_UNSUPPORTED_CONFIG, "LoRA rank must be <= 256");
        require(rows > 0 && cols > 0 && cols % 8 == 0, G4Q_ERR_INVALID_ARGUMENT,
                "rows must be > 0 and cols a positive multiple of 8");
        require(max_tokens >= 1 && max_tokens <= 65536, G4Q_ERR_INVALID_ARGUMENT, "max_tokens must be in [1, 65536]");
        require(lora_a != nullptr && lora_b != nullptr, G4Q_ERR_INVALID_ARGUMENT, "lora_a and lora_b must be non-null");
        auto* l = new (std::nothrow) Lora();
        require(l != nullptr, G4Q_ERR_MEMORY_GUARD, "host allocation failed");
        l->N = rows;
        l->K = cols;
        l->rank = rank;
        l->max_tokens = max_tokens;
        l->alpha = alpha;
        l->scale_bf16 = round_to_bf16(alpha / static_cast<float>(rank));
        l->device = current_device();
        float* b_tmp = nullptr;
        const size_t ab = (size_t)rank * cols * sizeof(float), bb = (size_t)rank * rows * sizeof(float);
        cudaError_t e = cudaMalloc(&l->a, ab);
        if (e == cudaSuccess) e = cudaMalloc(&l->bt, bb);
        if (e == cudaSuccess) e = cudaMalloc(&l->low, (size_t)max_tokens * rank * sizeof(float));
        if (e == cudaSuccess) e = cudaMalloc(&b_tmp, bb);
        if (e == cudaSuccess) e = cudaMemcpy(l->a, lora_a, ab, cudaMemcpyDefault);
        if (e == cudaSuccess) e = cudaMemcpy(b_tmp, lora_b, bb, cudaMemcpyDefault);
        if (e == cudaSuccess) {
            try {
                launch_lora_transpose(b_tmp, rows, rank, l->bt, nullptr);
            } catch (const Error&) {
                e = cudaErrorLaunchFailure;
            }
        }
        if (e == cudaSuccess) e = cudaDeviceSynchronize();
        cudaFree(b_tmp);
        if (e != cudaSuccess) {
            cudaFree(l->a);
            cudaFree(l->bt);
            cudaFree(l->low);
            delete l;
            check_cuda(e, "LoRA upload");
        }
        l->magic = kLoraMagic;
        *out = reinterpret_cast<G4qLora*>(l);
    });
}

G4qStatus g4q_lora_apply(const G4qLora* h, const uint16_t* x, int64_t M, int64_t ldx, uint16_t* y, int64_t ldy,
                         void* stream) {
    return guarded("g4q_lora_apply", [&] {
        Lora* l = checked_lora(h, "g4q_lora_apply");
        require(M >= 0, G4Q_ERR_INVALID_ARGUMENT, "M must be >= 0");
        if (M == 0) return;
        require(x != nullptr && y != nullptr, G4Q_ERR_INVALID_ARGUMENT, "x and y must be non-null");
        require(ldx >= l->K && ldx % 8 == 0, G4Q_ERR_INVALID_ARGUMENT, "ldx must be >= cols and a multiple of 8");
        require(ldy >= l->N, G4Q_ERR_INVALID_ARGUMENT, "ldy must be >= rows");
        require_aligned16(x, "x");
        require((reinterpret_cast<uintptr_t>(y) & 1u) == 0, G4Q_ERR_INVALID_ARGUMENT, "y must be 2-byte aligned");
        launch_lora_apply(*l, x, M, ldx, y, ldy, reinterpret_cast<cudaStream_t>(stream));
    });
}

G4qStatus g4q_lora_free(G4qLora* h) {
    return guarded("g4q_lora_free", [&] {
        auto* l = reinterpret_cast<Lora*>(h);
        require(l != nullptr, G4Q_ERR_INVALID_ARGUMENT, "requires a non-null LoRA handle");
        require(l->magic == kLoraMagic, G4Q_ERR_INVALID_ARGUMENT, "received an invalid LoRA handle");
        l->magic = 0;
        int prev = 0;
        cudaGetDevice(&prev);
        cudaSetDevice(l->device);
        cudaFree(l->a);
        cudaFree(l->bt);
        cudaFree(l->low);
        cudaSetDevice(prev);
        delete l;
    });
}

G4qStatus g4q_geglu(const uint16_t* gate, int64_t ld_gate, const uint16_t* up, int64_t ld_up, int64_t M, int64_t I,
                    uint16_t* out, int64_t ld_out, void* stream) {
    return guarded("g4q_geglu", [&] {
        require(M >= 0 && I >= 0 && I % 8 == 0, G4Q_ERR_INVALID_ARGUMENT, "M >= 0 and I a multiple of 8 are required");
        if (M == 0 || I == 0) return;
        require(gate != nullptr && up != nullptr && out != nullptr, G4Q_ERR_INVALID_ARGUMENT,
                "gate, up and out must be non-null");
        require(ld_gate >= I && ld_up >= I && ld_out >= I && ld_gate % 8 == 0 && ld_up % 8 == 0 && ld_out % 8 == 0,
                G4Q_ERR_INVALID_ARGUMENT, "row strides must be >= I and multiples of 8");
        require_aligned16(gate, "gate");
        require_aligned16(up, "up");
        require_aligned16(out, "out");
        launch_geglu(gate, ld_gate, up, ld_up, out, ld_out, M, I, reinterpret_cast<cudaStream_t>(stream));
    });
}

G4qStatus g4q_rms_norm(const uint16_t* x, int64_t ldx, const uint16_t* weight, int64_t M, int64_t K, float eps,
                       uint16_t* out, int64_t ld_out, void* stream) {
    return guarded("g4q_rms_norm", [&] {
        require(M >= 0 && K > 0 && K % 8 == 0, G4Q_ERR_INVALID_ARGUMENT, "M >= 0 and K a positive multiple of 8 are required");
        require(M <= 0x7FFFFFFF, G4Q_ERR_INVALID_ARGUMENT, "M must be < 2^31");
        if (M == 0) return;
        require(x != nullptr && out != nullptr, G4Q_ERR_INVALID_ARGUMENT, "x and out must be non-null");
        require(ldx >= K && ld_out >= K && ldx % 8 == 0 && ld_out % 8 == 0, G4Q_ERR_INVALID_ARGUMENT,
                "row strides must be >= K and multiples of 8");
        require(eps >= 0.0f && std::isfinite(eps), G4Q_ERR_INVALID_ARGUMENT, "eps must be finite and >= 0");
        require_aligned16(x, "x");
        require_aligned16(out, "out");
        if (weight != nullptr) require_aligned16(weight, "weight");
        launch_rms_norm(x, ldx, weight, M, K, eps, out, ld_out, reinterpret_cast<cudaStream_t>(stream));
    });
}

G4qStatus g4q_rms_norm_residual(const uint16_t* x, int64_t ldx, const uint16_t* weight, int64_t M, int64_t K,
                                float eps, const uint16_t* residual, int64_t ld_res, const uint16_t* layer_scalar,
                                uint16_t* out, int64_t ld_out, void* stream) {
    return guarded("g4q_rms_norm_residual", [&] {
        require(M >= 0 && K > 0 && K % 8 == 0, G4Q_ERR_INVALID_ARGUMENT, "M >= 0 and K a positive multiple of 8 are required");
        require(M <= 0x7FFFFFFF, G4Q_ERR_INVALID_ARGUMENT, "M must be < 2^31");
        if (M == 0) return;
        require(x != nullptr && residual != nullptr && out != nullptr, G4Q_ERR_INVALID_ARGUMENT,
                "x, residual and out must be non-null");
        require(ldx >= K && ld_res >= K && ld_out >= K && ldx % 8 == 0 && ld_res % 8 == 0 && ld_out % 8 == 0,
                G4Q_ERR_INVALID_ARGUMENT, "row strides must be >= K and multiples of 8");
        require(eps >= 0.0f && std::isfinite(eps), G4Q_ERR_INVALID_ARGUMENT, "eps must be finite and >= 0");
        require_aligned16(x, "x");
        require_aligned16(residual, "residual");
        require_aligned16(out, "out");
        if (weight != nullptr) require_aligned16(weight, "weight");
        launch_rms_norm(x, ldx, weight, M, K, eps, out, ld_out, reinterpret_cast<cudaStream_t>(stream), residual, ld_res,
                        layer_scalar);
    });
}

G4qStatus g4q_device_error(int32_t* code, int32_t reset) {
    return guarded("g4q_device_error", [&] {
        require(code != nullptr, G4Q_ERR_INVALID_ARGUMENT, "requires a non-null code pointer");
        // nothing is allocated here: a device on which only the allocation-free entry point ran
        // has no library scratch yet, and its error word is the entry point's static one
        int v = 0;
        if (DeviceScratch* ds = device_scratch_if_created()) {
            check_cuda(cudaMemcpy(&v, ds->err, sizeof(int), cudaMemcpyDeviceToHost), "read device error word");
            if (reset && v != 0) check_cuda(cudaMemset(ds->err, 0, sizeof(int)), "reset device error word");
        }
        const int v2 = noalloc_error(reset != 0);
        *code = v != 0 ? v : v2;
    });
}

G4qStatus g4q_synth_matrix(uint64_t seed, int64_t rows, int64_t cols, int32_t bits, int32_t group_size,
                           uint32_t* packed, uint16_t* scales, uint16_t* biases, void* stream) {
    return guarded("g4q_synth_matrix", [&] {
        require(bits == 4 || bits == 8, G4Q_ERR_UNSUPPORTED_CONFIG, "bits must be 4 or 8");
        require(group_size > 0 && cols % group_size == 0 && cols % (32 / bits) == 0, G4Q_ERR_INVALID_ARGUMENT,
                "cols must be a multiple of group_size");
        require(rows >= 0, G4Q_ERR_INVALID_ARGUMENT, "rows must be >= 0");
        require(scales != nullptr, G4Q_ERR_INVALID_ARGUMENT, "scales must be non-null");
        if (rows == 0) return;
        launch_synth_matrix(seed, rows, cols, bits, group_size, packed, scales, biases,
                            reinterpret_cast<cudaStream_t>(stream));
    });
}

G4qStatus g4q_synth_normal_bf16(uint64_t seed, int64_t count, uint16_t* out, void* stream) {
    return guarded("g4q_synth_normal_bf16", [&] {
        require(out != nullptr && count >= 0, G4Q_ERR_INVALID_ARGUMENT, "out must be non-null, count >= 0");
        if (count == 0) return;
        launch_synth_normal(seed, count, out, reinterpret_cast<cudaStream_t>(stream));
    });
}

}  // extern "C"
