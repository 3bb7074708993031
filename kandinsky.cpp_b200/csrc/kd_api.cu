// kd_api.cu -- the C ABI of libkd_attn (include/kd_attn.h): argument checks,
// the per-device context (scratch, error words, NCCL), TMA descriptors and
// the launch sequence of each entry point.  No CPU fallback anywhere: a shape
// the kernels do not cover is rejected with KD_ATTN_ERR_UNSUPPORTED.
#include <dlfcn.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <atomic>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/kd_attn.h"
#include "kd_internal.h"

using namespace kd;

struct kd_attn_ctx {
    int device = 0;
    int n_ranks = 1, rank = 0;
    kd_attn_log_cb log_cb = nullptr;
    void* log_user = nullptr;
    std::string last_error;
    unsigned* d_words = nullptr;  // [0] sticky error bits, [1] per-launch abort flag, [2] work counter,
                                  // [4..7] two u64 tile counters (K/V tiles loaded, tile products computed)
    void* scratch = nullptr;
    size_t scratch_bytes = 0;
    int num_sms = 148;
    void* nccl_comm = nullptr;
    unsigned long long wait_ns = 2000000000ull;  // bound on a single device-side wait
    // host-buffer pipeline (kd_attn_self_attention_host): copy streams and ordering events
    cudaStream_t h2d = nullptr, d2h = nullptr;
    cudaEvent_t ev_in[2] = {nullptr, nullptr}, ev_done[2] = {nullptr, nullptr}, ev_out[2] = {nullptr, nullptr};
    cudaEvent_t ev_start = nullptr, ev_last = nullptr;
    // head sharding: buffers allocated on every rank whose peers' copies are mapped here
    struct SymBuf {
        char* local = nullptr;
        size_t bytes = 0;
        char* peer[8] = {};  // indexed by rank; peer[rank] == local
    };
    std::vector<SymBuf> sym;
    unsigned char* d_barrier = nullptr;  // [64]: NCCL barrier send/receive bytes
};

namespace {

// ------------------------------------------------------------------ errors / logging
// Process-wide callback (kd_attn_set_log_callback) for contexts created without one and for
// calls that have no context.
std::mutex g_log_mu;
kd_attn_log_cb g_log_cb = nullptr;
void* g_log_user = nullptr;

void log_msg(kd_attn_ctx* ctx, kd_attn_log_level lvl, const char* fmt, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    if (ctx && ctx->log_cb) {
        ctx->log_cb(lvl, buf, ctx->log_user);
        return;
    }
    kd_attn_log_cb cb;
    void* user;
    {
        std::lock_guard<std::mutex> lock(g_log_mu);
        cb = g_log_cb;
        user = g_log_user;
    }
    if (cb)
        cb(lvl, buf, user);
    else if (lvl >= KD_ATTN_LOG_WARN)
        fprintf(stderr, "[kd_attn] %s\n", buf);
}

kd_attn_status fail(kd_attn_ctx* ctx, kd_attn_status st, const char* fmt, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    if (ctx) ctx->last_error = buf;
    log_msg(ctx, st == KD_ATTN_ERR_UNSUPPORTED ? KD_ATTN_LOG_WARN : KD_ATTN_LOG_ERROR, "%s", buf);
    return st;
}

#define KD_CUDA(ctx, call)                                                                              \
    do {                                                                                                \
        cudaError_t _e = (call);                                                                        \
        if (_e != cudaSuccess)                                                                          \
            return fail((ctx), KD_ATTN_ERR_CUDA, "%s failed: %s", #call, cudaGetErrorString(_e));      \
    } while (0)

struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

// ------------------------------------------------------------------ tensors
size_t elt_size(int32_t t) {
    switch (t) {
        case KD_ATTN_TYPE_F32: return 4;
        case KD_ATTN_TYPE_F16:
        case KD_ATTN_TYPE_BF16: return 2;
        default: return 0;
    }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ne[i] >= 0, sizes fit int, dim 0 contiguous.
kd_attn_status check_tensor(kd_attn_ctx* ctx, const kd_tensor* t, const char* name) {
    if (!t) return fail(ctx, KD_ATTN_ERR_INVALID_ARGUMENT, "%s is NULL", name);
    const size_t es = elt_size(t->type);
    if (!es) return fail(ctx, KD_ATTN_ERR_UNSUPPORTED, "%s: type %d is not f32/f16/bf16", name, t->type);
    for (int i = 0; i < 4; ++i)
        if (t->ne[i] < 0 || t->ne[i] > (int64_t)0x7fffffff)
            return fail(ctx, KD_ATTN_ERR_INVALID_ARGUMENT, "%s: ne[%d] = %lld out of range", name, i,
                        (long long)t->ne[i]);
    if (t->nb[0] != es) return fail(ctx, KD_ATTN_ERR_UNSUPPORTED, "%s: dim 0 must be contiguous", name);
    const bool empty = t->ne[0] == 0 || t->ne[1] == 0 || t->ne[2] == 0 || t->ne[3] == 0;
    if (!empty && !t->data) return fail(ctx, KD_ATTN_ERR_INVALID_ARGUMENT, "%s: data is NULL", name);
    return KD_ATTN_OK;
}

// Strides of size-1 dims are irrelevant; give them the packed value so TMA encoding accepts them.
void packed_strides(const kd_tensor* t, uint64_t nb[4]) {
    nb[0] = t->nb[0];
    for (int i = 1; i < 4; ++i) nb[i] = (t->ne[i] == 1) ? nb[i - 1] * (uint64_t)t->ne[i - 1] : t->nb[i];
}

bool strides16(const uint64_t nb[4]) { return nb[1] % 16 == 0 && nb[2] % 16 == 0 && nb[3] % 16 == 0; }

// ------------------------------------------------------------------ TMA descriptors
typedef CUresult (*PFN_encodeTiled_t)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                      const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                      CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

PFN_encodeTiled_t get_encode() {
    static PFN_encodeTiled_t fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_encodeTiled_t>(p);
    }
    return fn;
}

// [d, L, heads, seqs] 16-bit operand, {64, box_rows, 1, 1} box, 128-byte swizzle, zero fill out of range.
kd_attn_status make_operand_map(kd_attn_ctx* ctx, CUtensorMap* map, const void* data, bool bf16, int64_t L,
                                int64_t heads, int64_t seqs, const uint64_t nb[4], int64_t d = kHeadDim,
                                uint32_t box_rows = kBlockM) {
    PFN_encodeTiled_t enc = get_encode();
    if (!enc) return fail(ctx, KD_ATTN_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
    if (!aligned16(data)) return fail(ctx, KD_ATTN_ERR_UNSUPPORTED, "operand base address is not 16-byte aligned");
    cuuint64_t dims[4] = {(cuuint64_t)d, (cuuint64_t)(L > 0 ? L : 1), (cuuint64_t)(heads > 0 ? heads : 1),
                          (cuuint64_t)(seqs > 0 ? seqs : 1)};
    cuuint64_t strides[3] = {nb[1], nb[2], nb[3]};
    cuuint32_t box[4] = {64, box_rows, 1, 1};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    CUresult r = enc(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4,
                     const_cast<void*>(data), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(ctx, KD_ATTN_ERR_UNSUPPORTED, "cuTensorMapEncodeTiled rejected the operand (%d)", (int)r);
    return KD_ATTN_OK;
}

// The flash output [D, H, Lq, N] (16-bit) for TMA stores of 128-row O tiles: {64, 1, 128, 1} box,
// 128-byte swizzle.  Returns false (and the kernel stores rows directly) if the driver rejects it.
bool make_out_map(CUtensorMap* map, const void* data, int32_t type, int64_t D, int64_t H, int64_t Lq, int64_t N,
                  const uint64_t nb[4]) {
    PFN_encodeTiled_t enc = get_encode();
    if (!enc || !aligned16(data)) return false;
    cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)H, (cuuint64_t)Lq, (cuuint64_t)N};
    cuuint64_t strides[3] = {nb[1], nb[2], nb[3]};
    cuuint32_t box[4] = {64, 1, (cuuint32_t)kBlockM, 1};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    return enc(map, type == KD_ATTN_TYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4,
               const_cast<void*>(data), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
               CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// ------------------------------------------------------------------ scratch
size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

// Grows the context's scratch to at least `bytes`.  Growing happens on the first calls only.  The
// old buffer may still be read by work queued earlier: the context's calls are ordered on the
// call's stream (or by the caller's events into it, and the host-buffer copy streams are joined
// back into it), so draining that one stream is enough -- other streams of the device, such as a
// concurrent NCCL barrier, are not waited for.
kd_attn_status ensure_scratch(kd_attn_ctx* ctx, size_t bytes, cudaStream_t st) {
    if (bytes <= ctx->scratch_bytes) return KD_ATTN_OK;
    if (ctx->scratch) KD_CUDA(ctx, cudaStreamSynchronize(st));
    if (ctx->scratch) cudaFree(ctx->scratch);
    ctx->scratch = nullptr;
    ctx->scratch_bytes = 0;
    const size_t want = align256(bytes + bytes / 8);
    if (cudaMalloc(&ctx->scratch, want) != cudaSuccess) {
        cudaGetLastError();
        ctx->scratch = nullptr;
        return fail(ctx, KD_ATTN_ERR_OUT_OF_MEMORY, "could not allocate %zu bytes of scratch", want);
    }
    ctx->scratch_bytes = want;
    return KD_ATTN_OK;
}

// ------------------------------------------------------------------ NCCL (loaded on demand)
struct NcclUid {
    char internal[128];
};
struct Nccl {
    void* so = nullptr;
    int (*getUniqueId)(NcclUid*) = nullptr;
    int (*commInitRank)(void**, int, NcclUid, int) = nullptr;
    int (*allGather)(const void*, void*, size_t, int, void*, cudaStream_t) = nullptr;
    int (*commDestroy)(void*) = nullptr;
    const char* (*getErrorString)(int) = nullptr;
};

Nccl* nccl() {
    static Nccl n;
    static bool tried = false;
    if (!tried) {
        tried = true;
        const char* path = getenv("KD_ATTN_NCCL_LIB");
        n.so = dlopen(path && *path ? path : "libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (n.so) {
            n.getUniqueId = reinterpret_cast<int (*)(NcclUid*)>(dlsym(n.so, "ncclGetUniqueId"));
            n.commInitRank = reinterpret_cast<int (*)(void**, int, NcclUid, int)>(dlsym(n.so, "ncclCommInitRank"));
            n.allGather = reinterpret_cast<int (*)(const void*, void*, size_t, int, void*, cudaStream_t)>(
                dlsym(n.so, "ncclAllGather"));
            n.commDestroy = reinterpret_cast<int (*)(void*)>(dlsym(n.so, "ncclCommDestroy"));
            n.getErrorString = reinterpret_cast<const char* (*)(int)>(dlsym(n.so, "ncclGetErrorString"));
        }
    }
    if (!n.so || !n.getUniqueId || !n.commInitRank || !n.allGather || !n.commDestroy) return nullptr;
    return &n;
}
constexpr int kNcclUint8 = 1;  // ncclDataType_t ncclUint8

const char* nccl_err(Nccl* n, int r) { return (n && n->getErrorString) ? n->getErrorString(r) : "nccl error"; }

// Every rank of the group reaches this point of its stream before any passes it: one 1-byte
// all-gather on the context's communicator (a no-op for a single rank).
kd_attn_status rank_barrier(kd_attn_ctx* ctx, cudaStream_t st) {
    if (ctx->n_ranks <= 1) return KD_ATTN_OK;
    Nccl* n = nccl();
    if (!n || !ctx->nccl_comm) return fail(ctx, KD_ATTN_ERR_NCCL, "context has no NCCL communicator");
    const int r = n->allGather(ctx->d_barrier, ctx->d_barrier + 8, 1, kNcclUint8, ctx->nccl_comm, st);
    if (r != 0) return fail(ctx, KD_ATTN_ERR_NCCL, "ncclAllGather (barrier): %s", nccl_err(n, r));
    return KD_ATTN_OK;
}

// The symmetric buffer holding [p, p + bytes), or null.
kd_attn_ctx::SymBuf* find_sym(kd_attn_ctx* ctx, const void* p, size_t bytes) {
    const char* c = static_cast<const char*>(p);
    for (auto& b : ctx->sym)
        if (c >= b.local && c + bytes <= b.local + b.bytes) return &b;
    return nullptr;
}

void release_sym(kd_attn_ctx* ctx, kd_attn_ctx::SymBuf& b) {
    for (int i = 0; i < ctx->n_ranks && i < 8; ++i)
        if (i != ctx->rank && b.peer[i]) cudaIpcCloseMemHandle(b.peer[i]);
    if (b.local) cudaFree(b.local);
    b = kd_attn_ctx::SymBuf{};
}

OutType out_type_of(int32_t t) {
    return t == KD_ATTN_TYPE_F32 ? OutType::F32 : (t == KD_ATTN_TYPE_BF16 ? OutType::BF16 : OutType::F16);
}

// ------------------------------------------------------------------ flash core
struct FlashArgs {
    const kd_tensor* q;
    const kd_tensor* k;
    const kd_tensor* v;
    const kd_tensor* mask;
    float scale;
    const int32_t* kv_len;
    kd_tensor* out;
    float* lse;
    const uint8_t* tile_mask;  // bit-packed 64x64 tile bitmap or null
    // head sharding: the output's byte offset from `out_base` is also written at peer_base[i] + offset
    const char* out_base = nullptr;
    char* const* peer_base = nullptr;
    int n_peers = 0;
};

// ------------------------------------------------------------------ allocation-free scratch
// kd_attn_flash_ext_noalloc: the flash_attn_ext sequence (Q rounding, mask tile
// classes, tcgen05 kernel) with every piece of scratch taken from statically
// sized device arrays defined in this file, for callers that cannot allocate.
constexpr size_t kNoAllocScratchBytes = KD_ATTN_NOALLOC_SCRATCH_BYTES;
constexpr int kNoAllocMaxDevices = 64;

// One copy per device, created when the module loads and kept until the process exits.
// Host code must not use these names as addresses: it asks cudaGetSymbolAddress.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];
static __device__ __align__(256) unsigned g_noalloc_words[4];  // [0] sticky error bits, [1] abort flag, [2] work counter

struct NoAllocDevice {
    std::atomic<bool> ready{false};
    char* scratch = nullptr;   // device address of g_noalloc_scratch on this device
    unsigned* words = nullptr; // device address of g_noalloc_words on this device
    int num_sms = 0;
};
std::mutex g_noalloc_mu;
NoAllocDevice g_noalloc_dev[kNoAllocMaxDevices];

// Once per device, with that device current: resolve the arrays' device addresses.  Later calls
// take the lock-free path (the acquire load pairs with the release store that publishes them).
kd_attn_status noalloc_setup(NoAllocDevice** out) {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return fail(nullptr, KD_ATTN_ERR_CUDA, "cudaGetDevice failed: %s", cudaGetErrorString(e));
    if (dev < 0 || dev >= kNoAllocMaxDevices)
        return fail(nullptr, KD_ATTN_ERR_UNSUPPORTED, "device ordinal %d beyond %d", dev, kNoAllocMaxDevices);
    NoAllocDevice& d = g_noalloc_dev[dev];
    if (d.ready.load(std::memory_order_acquire)) {
        *out = &d;
        return KD_ATTN_OK;
    }
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!d.ready.load(std::memory_order_relaxed)) {
        int major = 0, minor = 0, sms = 0;
        if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
            cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess ||
            cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
            return fail(nullptr, KD_ATTN_ERR_CUDA, "device %d attributes unavailable", dev);
        if (major != 10 || minor != 0)
            return fail(nullptr, KD_ATTN_ERR_UNSUPPORTED, "device %d is sm_%d%d; built for sm_100a only", dev, major,
                        minor);
        void* s = nullptr;
        void* w = nullptr;
        e = cudaGetSymbolAddress(&s, g_noalloc_scratch);
        if (e != cudaSuccess)
            return fail(nullptr, KD_ATTN_ERR_CUDA, "cudaGetSymbolAddress(scratch) failed: %s", cudaGetErrorString(e));
        e = cudaGetSymbolAddress(&w, g_noalloc_words);
        if (e != cudaSuccess)
            return fail(nullptr, KD_ATTN_ERR_CUDA, "cudaGetSymbolAddress(words) failed: %s", cudaGetErrorString(e));
        d.scratch = static_cast<char*>(s);
        d.words = static_cast<unsigned*>(w);
        d.num_sms = sms;
        d.ready.store(true, std::memory_order_release);
    }
    *out = &d;
    return KD_ATTN_OK;
}

// The allocation-free entry point runs on the current device and has no context tying its
// buffers to a device: every buffer it is given must be device (or managed) memory that the
// current device owns.  cudaPointerGetAttributes allocates nothing.
kd_attn_status noalloc_check_ptr(const void* p, const char* name) {
    if (!p) return KD_ATTN_OK;
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return fail(nullptr, KD_ATTN_ERR_CUDA, "cudaGetDevice failed: %s", cudaGetErrorString(e));
    cudaPointerAttributes a{};
    e = cudaPointerGetAttributes(&a, p);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return fail(nullptr, KD_ATTN_ERR_INVALID_ARGUMENT, "%s: not a CUDA pointer (%s)", name, cudaGetErrorString(e));
    }
    if (a.type != cudaMemoryTypeDevice && a.type != cudaMemoryTypeManaged)
        return fail(nullptr, KD_ATTN_ERR_INVALID_ARGUMENT, "%s is not device memory", name);
    if (a.type == cudaMemoryTypeDevice && a.device != dev)
        return fail(nullptr, KD_ATTN_ERR_INVALID_ARGUMENT, "%s lives on device %d but the current device is %d", name,
                    a.device, dev);
    return KD_ATTN_OK;
}

// The flash_attn_ext sequence: argument checks, Q rounding to the operand type when needed, tile
// classes from the mask and/or the tile bitmap, tensor maps, the tcgen05 kernel.  With a context
// the scratch and device words are the context's; without one (`ctx` null, the allocation-free
// entry point) they are the static arrays above and messages go to stderr.
kd_attn_status flash_run(kd_attn_ctx* ctx, const FlashArgs& a, cudaStream_t st) {
    kd_attn_status rc;
    if ((rc = check_tensor(ctx, a.q, "q")) || (rc = check_tensor(ctx, a.k, "k")) ||
        (rc = check_tensor(ctx, a.v, "v")) || (rc = check_tensor(ctx, a.out, "out")))
        return rc;
    const kd_tensor &q = *a.q, &k = *a.k, &v = *a.v, &o = *a.out;
    // head_dim 128 (CrossDiT pro and lite image), 64 (CrossDiT lite video) or 512 (the VAE mid block,
    // kd_fmha512.cu: no mask, no kv_len, no peers)
    const int64_t D = q.ne[0];
    if ((D != kHeadDim && D != kHeadDim64 && D != kHeadDim512) || k.ne[0] != D || v.ne[0] != D)
        return fail(ctx, KD_ATTN_ERR_UNSUPPORTED, "head_dim must be 64, 128 or 512 (q %lld, k %lld, v %lld)",
                    (long long)q.ne[0], (long long)k.ne[0], (long long)v.ne[0]);
    const bool d512 = D == kHeadDim512;
    if (d512 && (a.mask || a.kv_len || a.tile_mask || a.n_peers))
        return fail(ctx, KD_ATTN_ERR_UNSUPPORTED, "head_dim 512 takes no mask, kv_len, tile mask or peers");
    if (k.type != v.type || (k.type != KD_ATTN_TYPE_F16 && k.type != KD_ATTN_TYPE_BF16))
        return fail(ctx, KD_ATTN_ERR_UNSUPPORTED, "k and v must share type f16 or bf16");
    const int64_t Lq = q.ne[1], H = q.ne[2], N = q.ne[3];
    const int64_t Lk = k.ne[1], Hkv = k.ne[2], Nkv = k.ne[3];
    if (v.ne[1] != Lk || v.ne[2] != Hkv || v.ne[3] != Nkv)
        return fail(ctx, KD_ATTN_ERR_INVALID_ARGUMENT, "v shape differs from k");
    if (Hkv <= 0 || Nkv <= 0 || H % Hkv || N % Nkv)
        return fail(ctx, KD_ATTN_ERR_INVALID_ARGUMENT, "q heads/sequences (%lld, %lld) are not multiples of k's (%lld, %lld)",
                    (long long)H, (long long)N, (long long)Hkv, (long long)Nkv);
    if (o.ne[0] != D || o.ne[1] != H || o.ne[2] != Lq || o.ne[3] != N)
        return fail(ctx, KD_ATTN_ERR_INVALID_ARGUMENT, "out must be [D, H, Lq, N]");
    if (d512 && Lk == 0 && Lq > 0)
        return fail(ctx, KD_ATTN_ERR_UNSUPPORTED, "head_dim 512 needs at least one key");
    if (!(a.scale > 0.f) || !std::isfinite(a.scale))
        return fail(ctx, KD_ATTN_ERR_UNSUPPORTED, "scale must be positive and finite");
    if (Lk > (int64_t)kMaxKvTiles * kBlockN)
        return fail(ctx, KD_ATTN_ERR_UNSUPPORTED, "Lk %lld exceeds %d", (long long)Lk, kMaxKvTiles * kBlockN);
    if (H > 65535 || N > 65535) return fail(ctx, KD_ATTN_ERR_UNSUPPORTED, "more than 65535 heads or sequences");
    uint64_t onb[4], knb[4], vnb[4], qnb[4];
    packed_strides(&o, onb);
    packed_strides(&k, knb);
    packed_strides(&v, vnb);
    packed_strides(&q, qnb);
    if (!strides16(onb) || !aligned16(o.data))
        return fail(ctx, KD_ATTN_ERR_UNSUPPORTED, "out rows must be 16-byte aligned");
    if (Lk > 0 && (!strides16(knb) || !strides16(vnb)))
        return fail(ctx, KD_ATTN_ERR_UNSUPPORTED, "k/v strides must be multiples of 16 bytes");
    if (Lq == 0 || H == 0 || N == 0) return KD_ATTN_OK;
    const bool bf16 = k.type == KD_ATTN_TYPE_BF16;

    // scratch plan: [Q rounded to the operand type][tile classes]
    const bool q_direct = q.type == k.type && strides16(qnb) && aligned16(q.data);
    const size_t q_bytes = q_direct ? 0 : align256((size_t)N * H * Lq * D * 2);
    const bool tiled = a.mask || a.tile_mask;
    const int n_qb = tiled ? (int)((Lq + 63) / 64) : 0, n_kb = tiled ? (int)((Lk + 63) / 64) : 0;
    int mh = 1, mn = 1;
    uint64_t mnb[4] = {0, 0, 0, 0};
    if (a.mask) {
        if ((rc = check_tensor(ctx, a.mask, "mask"))) return rc;
        const kd_tensor& m = *a.mask;
        if (m.type != KD_ATTN_TYPE_F16) return fail(ctx, KD_ATTN_ERR_UNSUPPORTED, "mask must be f16");
        if (m.ne[0] < Lk || m.ne[1] < Lq)
            return fail(ctx, KD_ATTN_ERR_INVALID_ARGUMENT, "mask [%lld, %lld] smaller than [Lk, Lq] = [%lld, %lld]",
                        (long long)m.ne[0], (long long)m.ne[1], (long long)Lk, (long long)Lq);
        if (m.ne[2] <= 0 || m.ne[3] <= 0 || H % m.ne[2] || N % m.ne[3])
            return fail(ctx, KD_ATTN_ERR_INVALID_ARGUMENT, "mask planes must divide heads and sequences");
        mh = (int)m.ne[2];
        mn = (int)m.ne[3];
        packed_strides(a.mask, mnb);
    }
    const size_t cls_bytes = tiled ? align256((size_t)mh * mn * n_qb * n_kb) : 0;

    char* scr = nullptr;
    unsigned* words = nullptr;
    unsigned long long* stats = nullptr;
    int num_sms = 0;
    unsigned long long wait_ns = 2000000000ull;
    if (ctx) {
        if ((rc = ensure_scratch(ctx, q_bytes + cls_bytes, st))) return rc;
        scr = static_cast<char*>(ctx->scratch);
        words = ctx->d_words;
        stats = reinterpret_cast<unsigned long long*>(ctx->d_words + 4);
        num_sms = ctx->num_sms;
        wait_ns = ctx->wait_ns;
    } else {
        if (q_bytes + cls_bytes > kNoAllocScratchBytes)
            return fail(ctx, KD_ATTN_ERR_UNSUPPORTED,
                        "kd_attn_flash_ext_noalloc needs %zu bytes of scratch but holds %zu "
                        "(KD_ATTN_NOALLOC_SCRATCH_BYTES); pass Q in K's type with 16-byte-aligned rows, or use "
                        "kd_attn_flash_ext",
                        q_bytes + cls_bytes, kNoAllocScratchBytes);
        if ((rc = noalloc_check_ptr(q.data, "q")) || (rc = noalloc_check_ptr(k.data, "k")) ||
            (rc = noalloc_check_ptr(v.data, "v")) || (rc = noalloc_check_ptr(o.data, "out")) ||
            (rc = noalloc_check_ptr(a.mask ? a.mask->data : nullptr, "mask")) ||
            (rc = noalloc_check_ptr(a.lse, "lse")) || (rc = noalloc_check_ptr(a.kv_len, "kv_len")) ||
            (rc = noalloc_check_ptr(a.tile_mask, "tile_mask")))
            return rc;
        NoAllocDevice* d = nullptr;
        if ((rc = noalloc_setup(&d))) return rc;
        scr = d->scratch;
        words = d->words;
        num_sms = d->num_sms;
    }

    const void* qdata = q.data;
    if (!q_direct) {
        ConvertParams cp{};
        cp.src = q.data;
        cp.src_type = q.type;
        cp.nb1 = (long long)qnb[1];
        cp.nb2 = (long long)qnb[2];
        cp.nb3 = (long long)qnb[3];
        cp.dst = scr;
        cp.L = (int)Lq;
        cp.H = (int)H;
        cp.N = (int)N;
        cp.D = (int)D;
        KD_CUDA(ctx, launch_convert_q(bf16 ? OpType::BF16 : OpType::F16, cp, num_sms, st));
        qdata = scr;
        qnb[1] = (uint64_t)D * 2;
        qnb[2] = qnb[1] * Lq;
        qnb[3] = qnb[2] * H;
    }
    uint8_t* cls = nullptr;
    if (tiled) {
        cls = reinterpret_cast<uint8_t*>(scr + q_bytes);
        MaskClassParams mp{};
        mp.mask = a.mask ? static_cast<const uint16_t*>(a.mask->data) : nullptr;
        mp.bits = a.tile_mask;
        mp.bits_row_bytes = (n_kb + 7) / 8;
        mp.vec16 = (a.mask && aligned16(a.mask->data) && mnb[1] % 16 == 0 && mnb[2] % 16 == 0 && mnb[3] % 16 == 0) ? 1 : 0;
        mp.nb1 = (long long)mnb[1];
        mp.nb2 = (long long)mnb[2];
        mp.nb3 = (long long)mnb[3];
        mp.Lq = (int)Lq;
        mp.Lk = (int)Lk;
        mp.mh = mh;
        mp.mn = mn;
        mp.cls = cls;
        mp.n_qb = n_qb;
        mp.n_kb = n_kb;
        KD_CUDA(ctx, launch_mask_classify(mp, st));  // writes every class byte
    }

    CUtensorMap tmQ, tmK, tmV;
    if (d512) {
        if ((rc = make_operand_map(ctx, &tmQ, qdata, bf16, Lq, H, N, qnb, D, 128)) ||
            (rc = make_operand_map(ctx, &tmK, k.data, bf16, Lk, Hkv, Nkv, knb, D, 64)) ||
            (rc = make_operand_map(ctx, &tmV, v.data, bf16, Lk, Hkv, Nkv, vnb, D, 64)))
            return rc;
        FmhaParams p{};
        p.Lq = (int)Lq;
        p.Lk = (int)Lk;
        p.H = (int)H;
        p.N = (int)N;
        p.rk2 = (int)(H / Hkv);
        p.rk3 = (int)(N / Nkv);
        p.scale_log2 = a.scale * 1.4426950408889634f;
        p.out = o.data;
        p.o_nb1 = (long long)onb[1];
        p.o_nb2 = (long long)onb[2];
        p.o_nb3 = (long long)onb[3];
        p.lse = a.lse;
        p.err = words;
        p.abort_flag = words + 1;
        p.wait_ns = wait_ns;
        KD_CUDA(ctx, cudaMemsetAsync(words + 1, 0, sizeof(unsigned), st));
        KD_CUDA(ctx, launch_fmha512(bf16 ? OpType::BF16 : OpType::F16, out_type_of(o.type), tmQ, tmK, tmV, p, st));
        return KD_ATTN_OK;
    }
    if ((rc = make_operand_map(ctx, &tmQ, qdata, bf16, Lq, H, N, qnb, D))) return rc;
    if (Lk > 0) {
        if ((rc = make_operand_map(ctx, &tmK, k.data, bf16, Lk, Hkv, Nkv, knb, D))) return rc;
        if ((rc = make_operand_map(ctx, &tmV, v.data, bf16, Lk, Hkv, Nkv, vnb, D))) return rc;
    } else {
        tmK = tmQ;  // never dereferenced: no key tiles to visit
        tmV = tmQ;
    }

    FmhaParams p{};
    p.D = (int)D;
    p.Lq = (int)Lq;
    p.Lk = (int)Lk;
    p.H = (int)H;
    p.N = (int)N;
    p.rk2 = (int)(H / Hkv);
    p.rk3 = (int)(N / Nkv);
    p.scale_log2 = a.scale * 1.4426950408889634f;
    p.inv_scale = 1.0f / a.scale;
    p.out = o.data;
    p.o_nb1 = (long long)onb[1];
    p.o_nb2 = (long long)onb[2];
    p.o_nb3 = (long long)onb[3];
    p.lse = a.lse;
    p.tile_cls = cls;
    p.n_qb = n_qb;
    p.n_kb = n_kb;
    if (a.mask) {
        p.mask = static_cast<const uint16_t*>(a.mask->data);
        p.m_nb1 = (long long)mnb[1];
        p.m_nb2 = (long long)mnb[2];
        p.m_nb3 = (long long)mnb[3];
    }
    p.mh = mh;
    p.mn = mn;
    p.kv_len = a.kv_len;
    p.err = words;
    p.abort_flag = words + 1;
    p.work_counter = words + 2;
    p.num_ctas = num_sms;
    p.wait_ns = wait_ns;
    p.tile_stats = stats;
    if (a.n_peers > kMaxPeers) return fail(ctx, KD_ATTN_ERR_UNSUPPORTED, "more than %d peers", kMaxPeers);
    for (int i = 0; i < a.n_peers; ++i)
        p.peer_out[i] = a.peer_base[i] + (static_cast<const char*>(o.data) - a.out_base);
    p.n_peer_out = a.n_peers;
    p.head_pairs = (tiled && mh == 1 && H % 2 == 0 && a.n_peers == 0) ? 1 : 0;
    p.out_v8 = (reinterpret_cast<uintptr_t>(o.data) % 32 == 0 && onb[1] % 32 == 0 && onb[2] % 32 == 0 &&
                onb[3] % 32 == 0) ? 1 : 0;
    // short-key calls (the kernel's double-buffered-Q instantiation) with a 16-bit output that is not
    // exchanged with peers write their O tiles with TMA stores
    CUtensorMap tmO = tmQ;  // never dereferenced unless p.tma_out
    p.tma_out = 0;
    if (!tiled && Lk > 0 && Lk <= kQ2MaxKeys && a.n_peers == 0 &&
        (o.type == KD_ATTN_TYPE_BF16 || o.type == KD_ATTN_TYPE_F16) &&
        make_out_map(&tmO, o.data, o.type, D, H, Lq, N, onb))
        p.tma_out = 1;
    // abort flag and work counter start at zero for every launch
    KD_CUDA(ctx, cudaMemsetAsync(words + 1, 0, 2 * sizeof(unsigned), st));
    KD_CUDA(ctx, launch_fmha(bf16 ? OpType::BF16 : OpType::F16, out_type_of(o.type), tmQ, tmK, tmV, tmO, p, st));
    return KD_ATTN_OK;
}

// ------------------------------------------------------------------ prologue core
// The RoPE table of one call: axes_dim must sum to the head dim D of the rotated tensors.
kd_attn_status fill_rope(kd_attn_ctx* ctx, const kd_rope3d* rope, int64_t L, int64_t D, RopeTab* tab) {
    const int a0 = rope->axes_dim[0], a1 = rope->axes_dim[1], a2 = rope->axes_dim[2];
    if (a0 < 0 || a1 < 0 || a2 < 0 || (a0 | a1 | a2) & 1 || a0 + a1 + a2 != D)
        return fail(ctx, KD_ATTN_ERR_INVALID_ARGUMENT, "rope axes_dim {%d,%d,%d} must be even and sum to the head dim %lld",
                    a0, a1, a2, (long long)D);
    const int64_t g = (int64_t)rope->grid[0] * rope->grid[1] * rope->grid[2];
    if (rope->grid[0] <= 0 || rope->grid[1] <= 0 || rope->grid[2] <= 0 || g != L)
        return fail(ctx, KD_ATTN_ERR_INVALID_ARGUMENT, "rope grid %dx%dx%d does not cover L = %lld", rope->grid[0],
                    rope->grid[1], rope->grid[2], (long long)L);
    for (int a = 0; a < 3; ++a)
        if (!(rope->scale_factor[a] > 0.f)) return fail(ctx, KD_ATTN_ERR_INVALID_ARGUMENT, "rope scale_factor must be > 0");
    if (!(rope->theta > 0.f)) return fail(ctx, KD_ATTN_ERR_INVALID_ARGUMENT, "rope theta must be > 0");
    const int halves[3] = {a0 / 2, a1 / 2, a2 / 2};
    int pi = 0;
    for (int a = 0; a < 3; ++a)
        for (int i = 0; i < halves[a]; ++i, ++pi) {
            // rope.hpp:23-29 get_freqs(dim = half): expf(-logf(theta) * i / dim), in float
            tab->freq[pi] = expf(-logf(rope->theta) * (float)i / (float)halves[a]);
            tab->div[pi] = rope->scale_factor[a];
            tab->axis[pi] = (unsigned char)a;
        }
    tab->grid_h = rope->grid[1];
    tab->grid_w = rope->grid[2];
    return KD_ATTN_OK;
}

// Checks one prologue tensor pair and fills its kernel description.  The head dim is
// D = x.ne[0] / n_head (as ops::attention derives it, ops.hpp:116): 128, or 64 (the lite models).
kd_attn_status prep_prologue_tensor(kd_attn_ctx* ctx, const kd_tensor* x, int32_t n_head, int32_t norm,
                                    const float* gain, bool rope, const kd_tensor* y, PrologueJob* t, int64_t* D_out) {
    kd_attn_status rc;
    if ((rc = check_tensor(ctx, x, "x")) || (rc = check_tensor(ctx, y, "y"))) return rc;
    if (x->type != KD_ATTN_TYPE_F32) return fail(ctx, KD_ATTN_ERR_UNSUPPORTED, "prologue input must be f32");
    const int64_t D = n_head > 0 ? x->ne[0] / n_head : 0;
    if (n_head <= 0 || (D != kHeadDim && D != kHeadDim64) || x->ne[0] != (int64_t)n_head * D)
        return fail(ctx, KD_ATTN_ERR_UNSUPPORTED, "x.ne[0] = %lld is not n_head * 128 or n_head * 64",
                    (long long)x->ne[0]);
    if (x->ne[3] != 1) return fail(ctx, KD_ATTN_ERR_INVALID_ARGUMENT, "x must be [C, L, N] (ne[3] == 1)");
    const int64_t L = x->ne[1], N = x->ne[2];
    if (y->ne[0] != D || y->ne[1] != L || y->ne[2] != n_head || y->ne[3] != N)
        return fail(ctx, KD_ATTN_ERR_INVALID_ARGUMENT, "y must be [D, L, n_head, N]");
    *D_out = D;
    if (L > INT32_MAX || N > INT32_MAX) return fail(ctx, KD_ATTN_ERR_UNSUPPORTED, "L or N beyond 2^31");
    uint64_t xnb[4], ynb[4];
    packed_strides(x, xnb);
    packed_strides(y, ynb);
    if (!aligned16(x->data) || xnb[1] % 16 || xnb[2] % 16)
        return fail(ctx, KD_ATTN_ERR_UNSUPPORTED, "x rows must be 16-byte aligned");
    const size_t ye = elt_size(y->type);
    if ((reinterpret_cast<uintptr_t>(y->data) % (4 * ye)) || ynb[1] % (4 * ye) || ynb[2] % (4 * ye) ||
        ynb[3] % (4 * ye))
        return fail(ctx, KD_ATTN_ERR_UNSUPPORTED, "y rows must be aligned to 4 elements");
    if (norm && gain && !aligned16(gain)) return fail(ctx, KD_ATTN_ERR_UNSUPPORTED, "gain must be 16-byte aligned");
    *t = PrologueJob{};
    t->x = static_cast<const float*>(x->data);
    t->x_nb1 = (long long)xnb[1];
    t->x_nb2 = (long long)xnb[2];
    t->y = y->data;
    t->y_nb1 = (long long)ynb[1];
    t->y_nb2 = (long long)ynb[2];
    t->y_nb3 = (long long)ynb[3];
    t->norm = norm ? 1 : 0;
    t->gain = norm ? gain : nullptr;
    t->rope = rope ? 1 : 0;
    t->L = (int)L;
    t->N = (int)N;
    t->H = n_head;
    return KD_ATTN_OK;
}

// One prologue launch over up to three projections (blockIdx.y = projection).  A RoPE grid must
// cover the L of every projection it rotates.
struct PrologueReq {
    const kd_tensor* x;
    int32_t norm;
    const float* gain;
    bool rope;
    const kd_tensor* y;
};

kd_attn_status prologue_multi(kd_attn_ctx* ctx, const PrologueReq* req, int count, int32_t n_head, float eps,
                              const kd_rope3d* rope, cudaStream_t st) {
    kd_attn_status rc;
    PrologueParams p{};
    p.eps = eps;
    int32_t ytype = -1;
    int64_t rope_L = -1;
    for (int i = 0; i < count; ++i) {
        PrologueJob t;
        const bool r = rope && req[i].rope;
        int64_t D = 0;
        if ((rc = prep_prologue_tensor(ctx, req[i].x, n_head, req[i].norm, req[i].gain, r, req[i].y, &t, &D)))
            return rc;
        if (p.D && D != p.D) return fail(ctx, KD_ATTN_ERR_INVALID_ARGUMENT, "prologue tensors of different head dims");
        p.D = (int)D;
        if (ytype >= 0 && req[i].y->type != ytype)
            return fail(ctx, KD_ATTN_ERR_INVALID_ARGUMENT, "prologue outputs must share one type");
        ytype = req[i].y->type;
        if (r) {
            if (rope_L >= 0 && rope_L != t.L)
                return fail(ctx, KD_ATTN_ERR_INVALID_ARGUMENT, "RoPE applied to tensors of different lengths");
            if (rope_L < 0 && (rc = fill_rope(ctx, rope, t.L, D, &p.tab))) return rc;
            rope_L = t.L;
        }
        if ((int64_t)t.L * t.N == 0) continue;
        p.job[p.njobs++] = t;
    }
    if (p.njobs == 0) return KD_ATTN_OK;
    KD_CUDA(ctx, launch_prologue(out_type_of(ytype), p, ctx->num_sms, st));
    return KD_ATTN_OK;
}

kd_attn_status prologue_core(kd_attn_ctx* ctx, const kd_tensor* x, int32_t n_head, int32_t norm, const float* gain,
                             float eps, const kd_rope3d* rope, kd_tensor* y, cudaStream_t st) {
    const PrologueReq r{x, norm, gain, rope != nullptr, y};
    return prologue_multi(ctx, &r, 1, n_head, eps, rope, st);
}

kd_tensor operand_view(void* data, int32_t type, int64_t L, int64_t H, int64_t N, int64_t D = kHeadDim) {
    kd_tensor t{};
    t.data = data;
    t.type = type;
    t.ne[0] = D;
    t.ne[1] = L;
    t.ne[2] = H;
    t.ne[3] = N;
    t.nb[0] = elt_size(type);
    t.nb[1] = t.nb[0] * D;
    t.nb[2] = t.nb[1] * (size_t)L;
    t.nb[3] = t.nb[2] * (size_t)H;
    return t;
}

// out [C, Lq, N] viewed as the flash dst [D, H, Lq, N]
kd_attn_status out_view(kd_attn_ctx* ctx, const kd_tensor* out, int32_t n_head, int64_t Lq, int64_t N, kd_tensor* v,
                        int64_t D = kHeadDim) {
    kd_attn_status rc;
    if ((rc = check_tensor(ctx, out, "out"))) return rc;
    if (out->ne[0] != (int64_t)n_head * D || out->ne[1] != Lq || out->ne[2] != N || out->ne[3] != 1)
        return fail(ctx, KD_ATTN_ERR_INVALID_ARGUMENT, "out must be [n_head*D, Lq, N] (D = %lld)", (long long)D);
    *v = *out;
    v->ne[0] = D;
    v->ne[1] = n_head;
    v->ne[2] = Lq;
    v->ne[3] = N;
    v->nb[1] = out->nb[0] * D;
    v->nb[2] = out->nb[1];
    v->nb[3] = out->nb[2];
    return KD_ATTN_OK;
}

// ops::attention with ONE head of 512 channels: VAEAttnBlock::forward (vae.hpp:89) on the H*W latent
// positions, no RMSNorm or RoPE.  The prologue (permute + rounding, 128-wide rows) takes each packed
// 512-wide row as four consecutive 128-wide rows, which lays the operands out as [512, L, 1, N];
// then the head_dim-512 flash kernel with scale 1/sqrt(512) (ops.hpp:161).
kd_attn_status attention512_core(kd_attn_ctx* ctx, const kd_tensor* q_in, const kd_tensor* k_in, const kd_tensor* v_in,
                                 const kd_tensor* mask, int32_t op_type, kd_tensor* out, float* lse, cudaStream_t st) {
    kd_attn_status rc;
    if (mask) return fail(ctx, KD_ATTN_ERR_UNSUPPORTED, "head_dim 512 takes no mask");
    const kd_tensor* ins[3] = {q_in, k_in, v_in};
    for (const kd_tensor* t : ins)
        if (t->ne[0] != kHeadDim512 || t->type != KD_ATTN_TYPE_F32 || t->nb[1] != (size_t)kHeadDim512 * 4 ||
            t->ne[3] != 1)
            return fail(ctx, KD_ATTN_ERR_UNSUPPORTED, "head_dim 512 needs packed f32 rows [512, L, N]");
    const int64_t Lq = q_in->ne[1], N = q_in->ne[2], Lk = k_in->ne[1];
    if (k_in->ne[2] != N || v_in->ne[1] != Lk || v_in->ne[2] != N)
        return fail(ctx, KD_ATTN_ERR_INVALID_ARGUMENT, "q_in/k_in/v_in shapes disagree");
    if ((rc = check_tensor(ctx, out, "out"))) return rc;
    if (out->ne[0] != kHeadDim512 || out->ne[1] != Lq || out->ne[2] != N || out->ne[3] != 1)
        return fail(ctx, KD_ATTN_ERR_INVALID_ARGUMENT, "out must be [512, Lq, N]");
    const size_t qb = align256((size_t)N * Lq * kHeadDim512 * 2);
    const size_t kb = align256((size_t)N * Lk * kHeadDim512 * 2);
    if ((rc = ensure_scratch(ctx, qb + 2 * kb, st))) return rc;
    char* base = static_cast<char*>(ctx->scratch);
    char* dst[3] = {base, base + qb, base + qb + kb};
    const int64_t len[3] = {Lq, Lk, Lk};
    kd_tensor x4[3], y4[3], ops[3];
    PrologueReq req[3];
    for (int i = 0; i < 3; ++i) {
        x4[i] = *ins[i];  // [128, 4L, N]: row pieces 512 bytes apart
        x4[i].ne[0] = kHeadDim;
        x4[i].ne[1] = 4 * len[i];
        x4[i].nb[1] = (size_t)kHeadDim * 4;
        y4[i] = operand_view(dst[i], op_type, 4 * len[i], 1, N);
        ops[i] = y4[i];  // the same bytes as [512, L, 1, N]
        ops[i].ne[0] = kHeadDim512;
        ops[i].ne[1] = len[i];
        ops[i].nb[1] = (size_t)kHeadDim512 * 2;
        req[i] = PrologueReq{&x4[i], 0, nullptr, false, &y4[i]};
    }
    if ((rc = prologue_multi(ctx, req, 3, 1, 0.f, nullptr, st))) return rc;
    kd_tensor ov = *out;  // [512, Lq, N] as the flash dst [512, 1, Lq, N]
    ov.ne[1] = 1;
    ov.ne[2] = Lq;
    ov.ne[3] = N;
    ov.nb[1] = out->nb[0] * kHeadDim512;
    ov.nb[2] = out->nb[1];
    ov.nb[3] = out->nb[2];
    FlashArgs fa{&ops[0], &ops[1], &ops[2], nullptr, 1.0f / std::sqrt((float)kHeadDim512), nullptr, &ov, lse};
    return flash_run(ctx, fa, st);
}

kd_attn_status attention_core(kd_attn_ctx* ctx, const kd_tensor* q_in, const kd_tensor* k_in, const kd_tensor* v_in,
                              int32_t n_head, const float* q_gain, const float* k_gain, float eps,
                              const kd_rope3d* rope, const kd_tensor* mask, const int32_t* kv_len, int32_t op_type,
                              kd_tensor* out, float* lse, cudaStream_t st, const char* out_base = nullptr,
                              char* const* peer_base = nullptr, int n_peers = 0, bool norm_qk = true) {
    kd_attn_status rc;
    if (n_head == 1 && q_in && q_in->ne[0] == kHeadDim512 && !norm_qk && !rope && !kv_len && !n_peers &&
        (op_type == KD_ATTN_TYPE_F16 || op_type == KD_ATTN_TYPE_BF16)) {
        if ((rc = check_tensor(ctx, q_in, "q_in")) || (rc = check_tensor(ctx, k_in, "k_in")) ||
            (rc = check_tensor(ctx, v_in, "v_in")))
            return rc;
        return attention512_core(ctx, q_in, k_in, v_in, mask, op_type, out, lse, st);
    }
    if ((rc = check_tensor(ctx, q_in, "q_in")) || (rc = check_tensor(ctx, k_in, "k_in")) ||
        (rc = check_tensor(ctx, v_in, "v_in")))
        return rc;
    if (op_type != KD_ATTN_TYPE_F16 && op_type != KD_ATTN_TYPE_BF16)
        return fail(ctx, KD_ATTN_ERR_UNSUPPORTED, "op_type must be f16 or bf16");
    const int64_t Lq = q_in->ne[1], N = q_in->ne[2], Lk = k_in->ne[1];
    if (k_in->ne[2] != N || v_in->ne[1] != Lk || v_in->ne[2] != N || v_in->ne[0] != k_in->ne[0])
        return fail(ctx, KD_ATTN_ERR_INVALID_ARGUMENT, "q_in/k_in/v_in shapes disagree");
    // head dim D = q_in.ne[0] / n_head (ops.hpp:116): 128, or 64 for the lite models
    const int64_t D = n_head > 0 ? q_in->ne[0] / n_head : 0;
    if (n_head <= 0 || (D != kHeadDim && D != kHeadDim64) || q_in->ne[0] != (int64_t)n_head * D)
        return fail(ctx, KD_ATTN_ERR_UNSUPPORTED, "q_in.ne[0] = %lld is not n_head * 128 or n_head * 64",
                    (long long)q_in->ne[0]);
    // K/V heads: k_in->ne[0] / D, a divisor of n_head (grouped-query attention, ops.hpp:135-157)
    if (k_in->ne[0] % D)
        return fail(ctx, KD_ATTN_ERR_UNSUPPORTED, "k_in.ne[0] = %lld is not a multiple of %lld", (long long)k_in->ne[0],
                    (long long)D);
    const int64_t n_kv_head = k_in->ne[0] / D;
    if (n_kv_head <= 0 || n_head % n_kv_head)
        return fail(ctx, KD_ATTN_ERR_INVALID_ARGUMENT, "invalid GQA ratio n_head=%d n_kv_head=%lld", n_head,
                    (long long)n_kv_head);
    kd_tensor ov;
    if ((rc = out_view(ctx, out, n_head, Lq, N, &ov, D))) return rc;
    const size_t es = 2;
    const size_t qb = align256((size_t)N * n_head * Lq * D * es);
    const size_t kb = align256((size_t)N * n_kv_head * Lk * D * es);
    // operand scratch sits after the flash core's own scratch needs: reserve them up front
    const size_t flash_extra =
        mask ? align256((size_t)mask->ne[2] * mask->ne[3] * ((Lq + 63) / 64) * ((Lk + 63) / 64)) : 0;
    if ((rc = ensure_scratch(ctx, flash_extra + qb + 2 * kb, st))) return rc;
    // The flash core carves its scratch from the start of the buffer; operands go after it.
    char* base = static_cast<char*>(ctx->scratch) + flash_extra;
    kd_tensor Qs = operand_view(base, op_type, Lq, n_head, N, D);
    kd_tensor Ks = operand_view(base + qb, op_type, Lk, n_kv_head, N, D);
    kd_tensor Vs = operand_view(base + qb + kb, op_type, Lk, n_kv_head, N, D);
    const int32_t nq = norm_qk ? 1 : 0;
    if (n_kv_head == n_head) {
        const PrologueReq req[3] = {{q_in, nq, q_gain, true, &Qs}, {k_in, nq, k_gain, true, &Ks},
                                    {v_in, 0, nullptr, false, &Vs}};
        if ((rc = prologue_multi(ctx, req, 3, n_head, eps, rope, st))) return rc;
    } else {  // different head counts: Q in one launch, K and V in another
        const PrologueReq rq[1] = {{q_in, nq, q_gain, true, &Qs}};
        const PrologueReq rkv[2] = {{k_in, nq, k_gain, true, &Ks}, {v_in, 0, nullptr, false, &Vs}};
        if ((rc = prologue_multi(ctx, rq, 1, n_head, eps, rope, st))) return rc;
        if ((rc = prologue_multi(ctx, rkv, 2, (int32_t)n_kv_head, eps, rope, st))) return rc;
    }
    FlashArgs fa{&Qs, &Ks, &Vs, mask, 1.0f / std::sqrt((float)D), kv_len, &ov, lse};
    fa.out_base = out_base;
    fa.peer_base = peer_base;
    fa.n_peers = n_peers;
    return flash_run(ctx, fa, st);
}

kd_attn_status ensure_copy_streams(kd_attn_ctx* ctx) {
    if (ctx->h2d) return KD_ATTN_OK;
    KD_CUDA(ctx, cudaStreamCreateWithFlags(&ctx->h2d, cudaStreamNonBlocking));
    KD_CUDA(ctx, cudaStreamCreateWithFlags(&ctx->d2h, cudaStreamNonBlocking));
    for (int i = 0; i < 2; ++i) {
        KD_CUDA(ctx, cudaEventCreateWithFlags(&ctx->ev_in[i], cudaEventDisableTiming));
        KD_CUDA(ctx, cudaEventCreateWithFlags(&ctx->ev_done[i], cudaEventDisableTiming));
        KD_CUDA(ctx, cudaEventCreateWithFlags(&ctx->ev_out[i], cudaEventDisableTiming));
    }
    KD_CUDA(ctx, cudaEventCreateWithFlags(&ctx->ev_start, cudaEventDisableTiming));
    KD_CUDA(ctx, cudaEventCreateWithFlags(&ctx->ev_last, cudaEventDisableTiming));
    return KD_ATTN_OK;
}

// Rows of a [C, L, N] host tensor restricted to columns [c0, c0 + width) <-> a packed device slab
// [width, L, N]: one 2-D copy when the sequences are evenly spaced, else one per sequence.
kd_attn_status copy_columns(kd_attn_ctx* ctx, const kd_tensor* host, size_t col_byte0, size_t width, void* dev,
                            bool to_device, cudaStream_t st) {
    const int64_t L = host->ne[1], N = host->ne[2];
    char* hbase = static_cast<char*>(host->data) + col_byte0;
    if (N == 1 || host->nb[2] == host->nb[1] * (size_t)L) {
        if (to_device)
            KD_CUDA(ctx, cudaMemcpy2DAsync(dev, width, hbase, host->nb[1], width, (size_t)(L * N), cudaMemcpyHostToDevice, st));
        else
            KD_CUDA(ctx, cudaMemcpy2DAsync(hbase, host->nb[1], dev, width, width, (size_t)(L * N), cudaMemcpyDeviceToHost, st));
        return KD_ATTN_OK;
    }
    for (int64_t n = 0; n < N; ++n) {
        char* h = hbase + n * host->nb[2];
        char* d = static_cast<char*>(dev) + (size_t)n * L * width;
        if (to_device)
            KD_CUDA(ctx, cudaMemcpy2DAsync(d, width, h, host->nb[1], width, (size_t)L, cudaMemcpyHostToDevice, st));
        else
            KD_CUDA(ctx, cudaMemcpy2DAsync(h, host->nb[1], d, width, width, (size_t)L, cudaMemcpyDeviceToHost, st));
    }
    return KD_ATTN_OK;
}

kd_attn_status self_attention_host(kd_attn_ctx* ctx, const kd_tensor* q_in, const kd_tensor* k_in,
                                   const kd_tensor* v_in, int32_t n_head, const float* q_gain, const float* k_gain,
                                   float eps, const kd_rope3d* rope, int32_t op_type, kd_tensor* out,
                                   cudaStream_t st) {
    kd_attn_status rc;
    if ((rc = check_tensor(ctx, q_in, "q_in")) || (rc = check_tensor(ctx, k_in, "k_in")) ||
        (rc = check_tensor(ctx, v_in, "v_in")) || (rc = check_tensor(ctx, out, "out")))
        return rc;
    if (q_in->type != KD_ATTN_TYPE_F32 || k_in->type != KD_ATTN_TYPE_F32 || v_in->type != KD_ATTN_TYPE_F32)
        return fail(ctx, KD_ATTN_ERR_UNSUPPORTED, "host inputs must be f32");
    const int64_t C = q_in->ne[0], L = q_in->ne[1], N = q_in->ne[2];
    for (const kd_tensor* t : {k_in, v_in})
        if (t->ne[0] != C || t->ne[1] != L || t->ne[2] != N || t->ne[3] != 1)
            return fail(ctx, KD_ATTN_ERR_INVALID_ARGUMENT, "q_in/k_in/v_in shapes disagree");
    const int64_t D = n_head > 0 ? C / n_head : 0;  // head dim: 128, or 64
    if (n_head <= 0 || (D != kHeadDim && D != kHeadDim64) || C != (int64_t)n_head * D || q_in->ne[3] != 1)
        return fail(ctx, KD_ATTN_ERR_UNSUPPORTED, "inputs must be [n_head*128, L, N] or [n_head*64, L, N]");
    if (out->ne[0] != C || out->ne[1] != L || out->ne[2] != N || out->ne[3] != 1)
        return fail(ctx, KD_ATTN_ERR_INVALID_ARGUMENT, "out must be [C, L, N] like the inputs");
    if (out->type != KD_ATTN_TYPE_F32 && out->type != op_type)
        return fail(ctx, KD_ATTN_ERR_UNSUPPORTED, "out must be f32 or the operand type");
    if (L * N == 0) return KD_ATTN_OK;
    // Group count: 4 to 16 groups of >= 64 MB of input each (only the last group's compute and
    // copy-out are exposed behind the copy-in); heads per group = the largest divisor of n_head
    // that gives at least that many groups.
    const size_t in_total = 3 * (size_t)C * 4 * (size_t)(L * N);
    const int want = (int)std::min<size_t>(16, std::max<size_t>(4, in_total / ((size_t)64 << 20)));
    int G = 1;
    for (int g = 1; g <= n_head; ++g)
        if (n_head % g == 0 && n_head / g >= want) G = g;
    // Group sizes: G heads each, except that the last G are split by halving (G/2, G/4, ..., 1, 1):
    // only the last group's compute and copy-out are exposed behind the (PCIe-bound) copy-in.
    std::vector<int> sizes;
    for (int g = 0; g < n_head / G - 1; ++g) sizes.push_back(G);
    for (int rest = n_head - (int)sizes.size() * G; rest > 0;) {
        const int part = std::min(G, rest > 1 ? (rest + 1) / 2 : 1);  // never more than a slab holds
        sizes.push_back(part);
        rest -= part;
    }
    const int groups = (int)sizes.size();
    const size_t in_w = (size_t)G * D * 4;                  // bytes per row of one input slab (max)
    const size_t out_es = elt_size(out->type);
    const size_t out_w = (size_t)G * D * out_es;
    const size_t in_slab = align256(in_w * (size_t)(L * N));
    const size_t out_slab = align256(out_w * (size_t)(L * N));
    const size_t opb = align256((size_t)N * G * L * D * 2);  // one operand for one group
    const size_t core = 3 * opb;                                     // attention_core's operand scratch
    if ((rc = ensure_copy_streams(ctx))) return rc;
    if ((rc = ensure_scratch(ctx, core + 2 * (3 * in_slab + out_slab), st))) return rc;
    char* stage = static_cast<char*>(ctx->scratch) + core;
    auto in_buf = [&](int b, int x) { return stage + ((size_t)b * 3 + x) * in_slab; };
    auto out_buf = [&](int b) { return stage + 6 * in_slab + (size_t)b * out_slab; };

    // the copies must not start before work already queued on the caller's stream
    KD_CUDA(ctx, cudaEventRecord(ctx->ev_start, st));
    KD_CUDA(ctx, cudaStreamWaitEvent(ctx->h2d, ctx->ev_start, 0));
    KD_CUDA(ctx, cudaStreamWaitEvent(ctx->d2h, ctx->ev_start, 0));
    const kd_tensor* ins[3] = {q_in, k_in, v_in};
    int head0 = 0;
    for (int g = 0; g < groups; head0 += sizes[g], ++g) {
        const int b = g & 1;
        const int gh = sizes[g];                                       // heads in this group
        const size_t gin_w = (size_t)gh * D * 4, gout_w = (size_t)gh * D * out_es;
        // inputs of group g go into slab b once group g-2's compute has finished with it
        if (g >= 2) KD_CUDA(ctx, cudaStreamWaitEvent(ctx->h2d, ctx->ev_done[b], 0));
        for (int x = 0; x < 3; ++x)
            if ((rc = copy_columns(ctx, ins[x], (size_t)head0 * D * 4, gin_w, in_buf(b, x), true, ctx->h2d)))
                return rc;
        KD_CUDA(ctx, cudaEventRecord(ctx->ev_in[b], ctx->h2d));
        // compute group g on the caller's stream; its output slab must have been copied out (group g-2)
        KD_CUDA(ctx, cudaStreamWaitEvent(st, ctx->ev_in[b], 0));
        if (g >= 2) KD_CUDA(ctx, cudaStreamWaitEvent(st, ctx->ev_out[b], 0));
        kd_tensor xs[3], os;
        for (int x = 0; x < 3; ++x) {
            xs[x] = *ins[x];
            xs[x].data = in_buf(b, x);
            xs[x].ne[0] = (int64_t)gh * D;
            xs[x].nb[1] = gin_w;
            xs[x].nb[2] = gin_w * (size_t)L;
            xs[x].nb[3] = xs[x].nb[2] * (size_t)N;
        }
        os = *out;
        os.data = out_buf(b);
        os.ne[0] = (int64_t)gh * D;
        os.nb[1] = gout_w;
        os.nb[2] = gout_w * (size_t)L;
        os.nb[3] = os.nb[2] * (size_t)N;
        if ((rc = attention_core(ctx, &xs[0], &xs[1], &xs[2], gh, q_gain, k_gain, eps, rope, nullptr, nullptr, op_type,
                                 &os, nullptr, st)))
            return rc;
        KD_CUDA(ctx, cudaEventRecord(ctx->ev_done[b], st));
        // copy group g's heads out into their columns of the host output
        KD_CUDA(ctx, cudaStreamWaitEvent(ctx->d2h, ctx->ev_done[b], 0));
        if ((rc = copy_columns(ctx, out, (size_t)head0 * D * out_es, gout_w, out_buf(b), false, ctx->d2h)))
            return rc;
        KD_CUDA(ctx, cudaEventRecord(ctx->ev_out[b], ctx->d2h));
    }
    // completion of the caller's stream covers the whole call (last copy-out included)
    KD_CUDA(ctx, cudaEventRecord(ctx->ev_last, ctx->d2h));
    KD_CUDA(ctx, cudaStreamWaitEvent(st, ctx->ev_last, 0));
    return KD_ATTN_OK;
}

// ------------------------------------------------------------------ QKV projection
// Bytes of one weight row of K elements (ggml_row_size).
int64_t weight_row_bytes(int32_t type, int64_t K) {
    switch (type) {
        case KD_ATTN_TYPE_F32: return K * 4;
        case KD_ATTN_TYPE_F16:
        case KD_ATTN_TYPE_BF16: return K * 2;
        case KD_ATTN_TYPE_Q8_0: return K / 32 * 34;
        case KD_ATTN_TYPE_Q4_0: return K / 32 * 18;
        default: return -1;
    }
}

// bf16 rows [rows] of Kp elements (Kp a multiple of kGemmKChunk), row_bytes apart, viewed as {64, rows, Kp/64}:
// a {64, box_rows, kGemmBoxChunks} box brings kGemmBoxChunks 64-wide K slices of box_rows rows, 128-byte
// swizzled; rows past the end read as zeros.
kd_attn_status make_gemm_map(kd_attn_ctx* ctx, CUtensorMap* map, const void* data, int64_t Kp, int64_t rows,
                             uint32_t box_rows, uint64_t row_bytes) {
    PFN_encodeTiled_t enc = get_encode();
    if (!enc) return fail(ctx, KD_ATTN_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
    cuuint64_t dims[3] = {64, (cuuint64_t)rows, (cuuint64_t)(Kp / 64)};
    cuuint64_t strides[2] = {(cuuint64_t)row_bytes, 128};
    cuuint32_t box[3] = {64, box_rows, (cuuint32_t)kGemmBoxChunks};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(data), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(ctx, KD_ATTN_ERR_UNSUPPORTED, "cuTensorMapEncodeTiled rejected a GEMM operand (%d)", (int)r);
    return KD_ATTN_OK;
}

// The GEMM's A operand: x [K, L, N] as M = L*N token rows.  f32 x is rounded into bf16 scratch rows of
// Kp elements; bf16 x whose K is a whole number of K steps and whose rows are evenly spaced and 16-byte
// aligned is read in place.
struct GemmInput {
    const kd_tensor* x = nullptr;
    int64_t K = 0, L = 0, N = 0, Kp = 0;
    uint64_t nb[4] = {};
    bool direct = false;  // bf16 rows read in place
};

kd_attn_status gemm_input(kd_attn_ctx* ctx, const kd_tensor* x, GemmInput* in) {
    kd_attn_status rc;
    if ((rc = check_tensor(ctx, x, "x"))) return rc;
    if (x->ne[3] != 1) return fail(ctx, KD_ATTN_ERR_INVALID_ARGUMENT, "x must be [K, L, N] (ne[3] == 1)");
    in->x = x;
    in->K = x->ne[0];
    in->L = x->ne[1];
    in->N = x->ne[2];
    if (in->K <= 0 || in->K % 32)
        return fail(ctx, KD_ATTN_ERR_UNSUPPORTED, "in_features %lld is not a positive multiple of 32", (long long)in->K);
    if (in->L * in->N > INT32_MAX - 256) return fail(ctx, KD_ATTN_ERR_UNSUPPORTED, "more than 2^31 tokens");
    in->Kp = (in->K + kGemmKChunk - 1) / kGemmKChunk * kGemmKChunk;  // rows zero-padded to whole K steps
    packed_strides(x, in->nb);
    if (!aligned16(x->data) || in->nb[1] % 16 || in->nb[2] % 16)
        return fail(ctx, KD_ATTN_ERR_UNSUPPORTED, "x rows must be 16-byte aligned");
    if (x->type == KD_ATTN_TYPE_BF16) {
        if (in->Kp != in->K || in->nb[2] != in->nb[1] * (uint64_t)in->L)
            return fail(ctx, KD_ATTN_ERR_UNSUPPORTED,
                        "bf16 x is read in place: K must be a multiple of %d and the sequences evenly spaced rows",
                        kGemmKChunk);
        in->direct = true;
    } else if (x->type != KD_ATTN_TYPE_F32) {
        return fail(ctx, KD_ATTN_ERR_UNSUPPORTED, "x must be f32 or bf16");
    }
    return KD_ATTN_OK;
}

// Checks one ggml Linear weight [K, C] (C a multiple of 256).
kd_attn_status check_weight(kd_attn_ctx* ctx, const kd_linear& W, int64_t K) {
    const int64_t rb = weight_row_bytes(W.type, K);
    if (rb < 0) return fail(ctx, KD_ATTN_ERR_UNSUPPORTED, "weight type %d is not f32/f16/bf16/q4_0/q8_0", W.type);
    if (W.ne[0] != K)
        return fail(ctx, KD_ATTN_ERR_INVALID_ARGUMENT, "weight ne[0] %lld != in_features %lld", (long long)W.ne[0],
                    (long long)K);
    if (W.ne[1] <= 0 || W.ne[1] % 256 || W.ne[1] > (1 << 20))
        return fail(ctx, KD_ATTN_ERR_UNSUPPORTED, "out_features %lld is not a multiple of 256 up to 2^20",
                    (long long)W.ne[1]);
    if ((int64_t)W.nb1 < rb) return fail(ctx, KD_ATTN_ERR_INVALID_ARGUMENT, "weight nb1 smaller than a row");
    if (!W.data) return fail(ctx, KD_ATTN_ERR_INVALID_ARGUMENT, "weight data is NULL");
    if ((W.type == KD_ATTN_TYPE_F32 || W.type == KD_ATTN_TYPE_F16 || W.type == KD_ATTN_TYPE_BF16) &&
        (!aligned16(W.data) || W.nb1 % 16))
        return fail(ctx, KD_ATTN_ERR_UNSUPPORTED, "f32/f16/bf16 weight rows must be 16-byte aligned");
    if (!aligned16(W.bias)) return fail(ctx, KD_ATTN_ERR_UNSUPPORTED, "bias must be 16-byte aligned");
    return KD_ATTN_OK;
}

// Scratch of one GEMM call: [B operand][A operand rows unless read in place][RoPE table].
size_t gemm_work_bytes(const GemmInput& in, int nslots, int64_t C, bool rot) {
    return align256((size_t)nslots * C * in.Kp * 2) + (in.direct ? 0 : align256((size_t)in.L * in.N * in.Kp * 2)) +
           (rot ? align256((size_t)in.L * (kHeadDim / 2) * sizeof(float2)) : 0);  // (at most 64 pairs per token)
}

// Launch sequence of one GEMM: each weight w[i] expanded to bf16 rows of the B operand (slot i = rows
// [i*C, (i+1)*C)); x rounded to bf16 token rows unless read in place; the RoPE (cos, sin) table when a slot
// rotates; then the persistent GEMM whose epilogue writes every slot's output.  `work` holds
// gemm_work_bytes(in, p.nslots, p.C, tab != nullptr) bytes.
kd_attn_status gemm_run(kd_attn_ctx* ctx, const GemmInput& in, const kd_linear* const* w, QkvParams& p,
                        const RopeTab* tab, int32_t out_dtype, char* work, cudaStream_t st) {
    kd_attn_status rc;
    const int64_t C = p.C, Kp = in.Kp;
    p.K = (int)in.K;
    p.L = (int)in.L;
    p.M = (int)(in.L * in.N);
    if (p.M == 0) return KD_ATTN_OK;
    const size_t b_bytes = align256((size_t)p.nslots * C * Kp * 2);
    const size_t a_bytes = in.direct ? 0 : align256((size_t)p.M * Kp * 2);
    __nv_bfloat16* wb = reinterpret_cast<__nv_bfloat16*>(work);
    for (int i = 0; i < p.nslots; ++i)
        KD_CUDA(ctx, launch_expand_weights(w[i]->data, w[i]->type, (long long)w[i]->nb1, (int)in.K, (int)Kp, (int)C,
                                           i * (int)C, wb, ctx->num_sms, st));
    const void* xa = in.x->data;
    uint64_t xrow = in.nb[1];
    if (!in.direct) {
        __nv_bfloat16* xb = reinterpret_cast<__nv_bfloat16*>(work + b_bytes);
        KD_CUDA(ctx, launch_to_bf16_rows(in.x->data, (long long)in.nb[1], (long long)in.nb[2], (int)in.K, (int)Kp,
                                         (int)in.L, p.M, xb, ctx->num_sms, st));
        xa = xb;
        xrow = (uint64_t)Kp * 2;
    }
    if (tab) {
        float2* cs = reinterpret_cast<float2*>(work + b_bytes + a_bytes);
        KD_CUDA(ctx, launch_rope_table(*tab, (int)in.L, p.D / 2, cs, ctx->num_sms, st));
        p.rope_cs = cs;
    }
    CUtensorMap tmX, tmW;
    if ((rc = make_gemm_map(ctx, &tmX, xa, Kp, p.M, kGemmBoxRowsA, xrow)) ||
        (rc = make_gemm_map(ctx, &tmW, wb, Kp, (int64_t)p.nslots * C, kGemmBoxRowsB, (uint64_t)Kp * 2)))
        return rc;
    p.err = ctx->d_words;
    p.abort_flag = ctx->d_words + 1;
    p.wait_ns = ctx->wait_ns;
    KD_CUDA(ctx, cudaMemsetAsync(ctx->d_words + 1, 0, sizeof(unsigned), st));
    KD_CUDA(ctx, launch_qkv_gemm(out_type_of(out_dtype), tmX, tmW, p, ctx->num_sms, st));
    return KD_ATTN_OK;
}

// to_query/to_key/to_value + prologue (see kd_attn_qkv_projection).  `work` = NULL: the context's scratch.
kd_attn_status qkv_projection_core(kd_attn_ctx* ctx, const kd_tensor* x, const kd_linear* const w[3],
                                   const float* q_gain, const float* k_gain, float eps, const kd_rope3d* rope,
                                   int32_t out_dtype, kd_tensor* const outs[3], cudaStream_t st, char* work = nullptr) {
    kd_attn_status rc;
    GemmInput in;
    if ((rc = gemm_input(ctx, x, &in))) return rc;
    if (in.x->type != KD_ATTN_TYPE_F32) return fail(ctx, KD_ATTN_ERR_UNSUPPORTED, "x must be f32");
    if (out_dtype != KD_ATTN_TYPE_F16 && out_dtype != KD_ATTN_TYPE_BF16)
        return fail(ctx, KD_ATTN_ERR_UNSUPPORTED, "the projection writes f16 or bf16 operands");
    const int64_t K = in.K, L = in.L, N = in.N;
    QkvParams p{};
    p.eps = eps;
    int64_t C = -1, D = -1;
    const kd_linear* ws[3] = {};
    for (int i = 0; i < 3; ++i) {
        if (!w[i] && !outs[i]) continue;
        if (!w[i] || !outs[i]) return fail(ctx, KD_ATTN_ERR_INVALID_ARGUMENT, "a weight and its output must both be given");
        const kd_linear& W = *w[i];
        const kd_tensor& o = *outs[i];
        if ((rc = check_tensor(ctx, &o, "projection output"))) return rc;
        if (o.type != out_dtype) return fail(ctx, KD_ATTN_ERR_INVALID_ARGUMENT, "outputs must have type out_dtype");
        if ((rc = check_weight(ctx, W, K))) return rc;
        if (C >= 0 && W.ne[1] != C) return fail(ctx, KD_ATTN_ERR_INVALID_ARGUMENT, "the weights disagree on out_features");
        C = W.ne[1];
        // head dim from the outputs: 128, or 64 (the lite video model)
        if (D >= 0 && o.ne[0] != D) return fail(ctx, KD_ATTN_ERR_INVALID_ARGUMENT, "outputs disagree on the head dim");
        D = o.ne[0];
        if (D != kHeadDim && D != kHeadDim64)
            return fail(ctx, KD_ATTN_ERR_UNSUPPORTED, "output head dim %lld is not 128 or 64", (long long)D);
        if (o.ne[1] != L || o.ne[2] * D != C || o.ne[3] != N)
            return fail(ctx, KD_ATTN_ERR_INVALID_ARGUMENT, "outputs must be [D, L, C/D, N]");
        uint64_t onb[4];
        packed_strides(&o, onb);
        if (!aligned16(o.data) || !strides16(onb))
            return fail(ctx, KD_ATTN_ERR_UNSUPPORTED, "output rows must be 16-byte aligned");
        QkvSlot& S = p.slot[p.nslots];
        S.out = o.data;
        S.o_nb1 = (long long)onb[1];
        S.o_nb2 = (long long)onb[2];
        S.o_nb3 = (long long)onb[3];
        S.bias = W.bias;
        S.norm = i < 2;
        S.gain = i == 0 ? q_gain : (i == 1 ? k_gain : nullptr);
        S.rope = (i < 2 && rope) ? 1 : 0;
        ws[p.nslots++] = w[i];
    }
    if (p.nslots == 0) return KD_ATTN_OK;
    if (!aligned16(q_gain) || !aligned16(k_gain))
        return fail(ctx, KD_ATTN_ERR_UNSUPPORTED, "q_gain / k_gain must be 16-byte aligned");
    p.C = (int)C;
    p.D = (int)D;
    RopeTab tab{};
    const bool rot = rope && (p.slot[0].rope || (p.nslots > 1 && p.slot[1].rope));
    if (rot && (rc = fill_rope(ctx, rope, L, D, &tab))) return rc;
    if (L * N == 0) return KD_ATTN_OK;
    if (!work) {
        if ((rc = ensure_scratch(ctx, gemm_work_bytes(in, p.nslots, C, rot), st))) return rc;
        work = static_cast<char*>(ctx->scratch);
    }
    return gemm_run(ctx, in, ws, p, rot ? &tab : nullptr, out_dtype, work, st);
}

// ops::linear (ops.hpp:27-42): y = x W^T + b.  x [K, L, N] f32 or bf16, y [C, L, N] f32 / bf16 / f16 with
// contiguous, 16-byte-aligned rows.  `work` = NULL: the context's scratch.
// ops::linear on the projection GEMM.
kd_attn_status linear_core(kd_attn_ctx* ctx, const kd_tensor* x, const kd_linear* w, kd_tensor* y, cudaStream_t st,
                           char* work = nullptr) {
    kd_attn_status rc;
    GemmInput in;
    if ((rc = gemm_input(ctx, x, &in))) return rc;
    if (!w) return fail(ctx, KD_ATTN_ERR_INVALID_ARGUMENT, "w is NULL");
    if ((rc = check_weight(ctx, *w, in.K))) return rc;
    if ((rc = check_tensor(ctx, y, "y"))) return rc;
    const int64_t C = w->ne[1];
    if (y->ne[0] != C || y->ne[1] != in.L || y->ne[2] != in.N || y->ne[3] != 1)
        return fail(ctx, KD_ATTN_ERR_INVALID_ARGUMENT, "y must be [out_features, L, N]");
    uint64_t ynb[4];
    packed_strides(y, ynb);
    if (!aligned16(y->data) || ynb[1] % 16 || ynb[2] % 16)
        return fail(ctx, KD_ATTN_ERR_UNSUPPORTED, "y rows must be 16-byte aligned");
    QkvParams p{};
    p.nslots = 1;
    p.C = (int)C;
    p.D = kHeadDim;  // no norm or RoPE: the output is addressed in 128-column groups
    QkvSlot& S = p.slot[0];
    // a row-major [C, L, N] output in the epilogue's (row, 128-column group, sequence) addressing
    S.out = y->data;
    S.o_nb1 = (long long)ynb[1];
    S.o_nb2 = (long long)(kHeadDim * elt_size(y->type));
    S.o_nb3 = (long long)ynb[2];
    S.bias = w->bias;
    if (in.L * in.N == 0) return KD_ATTN_OK;
    if (!work) {
        if ((rc = ensure_scratch(ctx, gemm_work_bytes(in, 1, C, false), st))) return rc;
        work = static_cast<char*>(ctx->scratch);
    }
    const kd_linear* ws[1] = {w};
    return gemm_run(ctx, in, ws, p, nullptr, y->type, work, st);
}

// DiTSelfAttention::forward (crossdit.hpp:117-154) from the hidden states: fused QKV projection, flash
// attention, out-projection.  Scratch: [Q][K][V operands][attention output][GEMM work, shared by both GEMMs].
// The head dim of a block whose projections map to C features over n_head heads (DiTSelfAttention's and
// DiTCrossAttention's num_heads, crossdit.hpp): D = C / n_head, 128 or 64.
kd_attn_status block_head_dim(kd_attn_ctx* ctx, const kd_linear* wq, const kd_linear* wk, const kd_linear* wv,
                              const kd_linear* wo, int32_t n_head, int64_t* D) {
    if (!wq || !wk || !wv || !wo) return fail(ctx, KD_ATTN_ERR_INVALID_ARGUMENT, "all four weights are required");
    const int64_t C = wq->ne[1];
    if (wk->ne[1] != C || wv->ne[1] != C || wo->ne[0] != C)
        return fail(ctx, KD_ATTN_ERR_INVALID_ARGUMENT, "the projections must map to C features and back");
    *D = n_head > 0 ? C / n_head : 0;
    if (n_head <= 0 || (*D != kHeadDim && *D != kHeadDim64) || (int64_t)n_head * *D != C)
        return fail(ctx, KD_ATTN_ERR_UNSUPPORTED, "C = %lld over %d heads is not a head dim of 128 or 64", (long long)C,
                    n_head);
    return KD_ATTN_OK;
}

kd_attn_status self_attention_block_core(kd_attn_ctx* ctx, const kd_tensor* x, const kd_linear* wq,
                                         const kd_linear* wk, const kd_linear* wv, const kd_linear* wo,
                                         int32_t n_head, const float* q_gain, const float* k_gain, float eps,
                                         const kd_rope3d* rope, kd_tensor* y, cudaStream_t st) {
    kd_attn_status rc;
    GemmInput in;
    if ((rc = gemm_input(ctx, x, &in))) return rc;
    int64_t D = 0;
    if ((rc = block_head_dim(ctx, wq, wk, wv, wo, n_head, &D))) return rc;
    const int64_t C = wq->ne[1], L = in.L, N = in.N;
    const int32_t H = n_head;
    const int32_t op = KD_ATTN_TYPE_BF16;
    const size_t opb = align256((size_t)N * H * L * D * 2);
    const bool rot = rope != nullptr;
    GemmInput attn_in = in;  // the out-projection reads the attention output [C, L, N] bf16 in place
    attn_in.K = attn_in.Kp = C;
    attn_in.direct = true;
    const size_t work = std::max(gemm_work_bytes(in, 3, C, rot), gemm_work_bytes(attn_in, 1, wo->ne[1], false));
    if ((rc = ensure_scratch(ctx, 4 * opb + work, st))) return rc;
    char* base = static_cast<char*>(ctx->scratch);
    kd_tensor Qs = operand_view(base, op, L, H, N, D);
    kd_tensor Ks = operand_view(base + opb, op, L, H, N, D);
    kd_tensor Vs = operand_view(base + 2 * opb, op, L, H, N, D);
    kd_tensor A{};  // attention output [C, L, N] bf16 = the flash dst [D, H, L, N]
    A.data = base + 3 * opb;
    A.type = op;
    A.ne[0] = C;
    A.ne[1] = L;
    A.ne[2] = N;
    A.ne[3] = 1;
    A.nb[0] = 2;
    A.nb[1] = 2 * (size_t)C;
    A.nb[2] = A.nb[1] * (size_t)L;
    A.nb[3] = A.nb[2] * (size_t)N;
    char* gw = base + 4 * opb;
    const kd_linear* w3[3] = {wq, wk, wv};
    kd_tensor* o3[3] = {&Qs, &Ks, &Vs};
    if ((rc = qkv_projection_core(ctx, x, w3, q_gain, k_gain, eps, rope, op, o3, st, gw))) return rc;
    kd_tensor ov;
    if ((rc = out_view(ctx, &A, H, L, N, &ov, D))) return rc;
    FlashArgs fa{&Qs, &Ks, &Vs, nullptr, 1.0f / std::sqrt((float)D), nullptr, &ov, nullptr};
    if ((rc = flash_run(ctx, fa, st))) return rc;  // bf16 operands, no mask: no scratch of its own
    return linear_core(ctx, &A, wo, y, st, gw);
}

// DiTCrossAttention::forward (crossdit.hpp:174-200) from the visual and text hidden states: the Q
// projection of x_query and the K/V projections of x_kv (RMSNorm on Q and K, no RoPE), the flash kernel
// with the text's valid lengths (kv_len and/or an f16 mask), the out-projection.  Scratch: [the flash
// core's mask-class scratch][Q][K][V operands][attention output][GEMM work shared by the three GEMMs].
kd_attn_status cross_attention_block_core(kd_attn_ctx* ctx, const kd_tensor* x_query, const kd_tensor* x_kv,
                                          const kd_linear* wq, const kd_linear* wk, const kd_linear* wv,
                                          const kd_linear* wo, int32_t n_head, const float* q_gain,
                                          const float* k_gain, float eps, const kd_tensor* mask,
                                          const int32_t* kv_len, kd_tensor* y, cudaStream_t st) {
    kd_attn_status rc;
    GemmInput iq, ikv;
    if ((rc = gemm_input(ctx, x_query, &iq)) || (rc = gemm_input(ctx, x_kv, &ikv))) return rc;
    int64_t D = 0;
    if ((rc = block_head_dim(ctx, wq, wk, wv, wo, n_head, &D))) return rc;
    const int64_t C = wq->ne[1], Lq = iq.L, Lk = ikv.L, N = iq.N;
    if (ikv.N != N) return fail(ctx, KD_ATTN_ERR_INVALID_ARGUMENT, "x_query and x_kv disagree on the batch");
    const int32_t H = n_head;
    const int32_t op = KD_ATTN_TYPE_BF16;
    const size_t qb = align256((size_t)N * H * Lq * D * 2);
    const size_t kb = align256((size_t)N * H * Lk * D * 2);
    const size_t flash_extra =
        mask ? align256((size_t)mask->ne[2] * mask->ne[3] * ((Lq + 63) / 64) * ((Lk + 63) / 64)) : 0;
    GemmInput attn_in = iq;  // the out-projection reads the attention output [C, Lq, N] bf16 in place
    attn_in.K = attn_in.Kp = C;
    attn_in.direct = true;
    const size_t work = std::max({gemm_work_bytes(iq, 1, C, false), gemm_work_bytes(ikv, 2, C, false),
                                  gemm_work_bytes(attn_in, 1, wo->ne[1], false)});
    if ((rc = ensure_scratch(ctx, flash_extra + 2 * qb + 2 * kb + work, st))) return rc;
    char* base = static_cast<char*>(ctx->scratch) + flash_extra;
    kd_tensor Qs = operand_view(base, op, Lq, H, N, D);
    kd_tensor Ks = operand_view(base + qb, op, Lk, H, N, D);
    kd_tensor Vs = operand_view(base + qb + kb, op, Lk, H, N, D);
    kd_tensor A{};  // attention output [C, Lq, N] bf16 = the flash dst [D, H, Lq, N]
    A.data = base + qb + 2 * kb;
    A.type = op;
    A.ne[0] = C;
    A.ne[1] = Lq;
    A.ne[2] = N;
    A.ne[3] = 1;
    A.nb[0] = 2;
    A.nb[1] = 2 * (size_t)C;
    A.nb[2] = A.nb[1] * (size_t)Lq;
    A.nb[3] = A.nb[2] * (size_t)N;
    char* gw = base + 2 * qb + 2 * kb;
    const kd_linear* wq3[3] = {wq, nullptr, nullptr};
    kd_tensor* oq3[3] = {&Qs, nullptr, nullptr};
    if ((rc = qkv_projection_core(ctx, x_query, wq3, q_gain, nullptr, eps, nullptr, op, oq3, st, gw))) return rc;
    const kd_linear* wkv3[3] = {nullptr, wk, wv};
    kd_tensor* okv3[3] = {nullptr, &Ks, &Vs};
    if ((rc = qkv_projection_core(ctx, x_kv, wkv3, nullptr, k_gain, eps, nullptr, op, okv3, st, gw))) return rc;
    kd_tensor ov;
    if ((rc = out_view(ctx, &A, H, Lq, N, &ov, D))) return rc;
    FlashArgs fa{&Qs, &Ks, &Vs, mask, 1.0f / std::sqrt((float)D), kv_len, &ov, nullptr};
    if ((rc = flash_run(ctx, fa, st))) return rc;
    return linear_core(ctx, &A, wo, y, st, gw);
}

}  // namespace

// ====================================================================== C ABI
extern "C" {

int32_t kd_attn_version(void) { return (KD_ATTN_VERSION_MAJOR << 16) | KD_ATTN_VERSION_MINOR; }

kd_attn_status kd_attn_nccl_unique_id(void* out128) {
    if (!out128) return KD_ATTN_ERR_INVALID_ARGUMENT;
    Nccl* n = nccl();
    if (!n) return fail(nullptr, KD_ATTN_ERR_NCCL, "NCCL could not be loaded (libnccl.so.2)");
    NcclUid id;
    const int r = n->getUniqueId(&id);
    if (r != 0) return fail(nullptr, KD_ATTN_ERR_NCCL, "ncclGetUniqueId: %s", nccl_err(n, r));
    memcpy(out128, id.internal, sizeof id.internal);
    return KD_ATTN_OK;
}

kd_attn_status kd_attn_create(const kd_attn_init* init, kd_attn_ctx** out) {
    if (!out) return KD_ATTN_ERR_INVALID_ARGUMENT;
    *out = nullptr;
    if (!init) return KD_ATTN_ERR_INVALID_ARGUMENT;
    if (init->n_ranks < 1 || init->rank < 0 || init->rank >= init->n_ranks) return KD_ATTN_ERR_INVALID_ARGUMENT;
    kd_attn_ctx* ctx = new kd_attn_ctx();
    ctx->device = init->device;
    ctx->n_ranks = init->n_ranks;
    ctx->rank = init->rank;
    ctx->log_cb = init->log_cb;
    ctx->log_user = init->log_user_data;
    if (const char* w = getenv("KD_ATTN_WAIT_MS")) {
        const long long ms = atoll(w);
        if (ms > 0) ctx->wait_ns = (unsigned long long)ms * 1000000ull;
    }
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || init->device < 0 || init->device >= ndev) {
        cudaGetLastError();
        fail(ctx, KD_ATTN_ERR_CUDA, "CUDA device %d is not available", init->device);
        delete ctx;
        return KD_ATTN_ERR_CUDA;
    }
    DeviceGuard g(ctx->device);
    cudaDeviceProp prop{};
    if (cudaGetDeviceProperties(&prop, ctx->device) != cudaSuccess) {
        delete ctx;
        return KD_ATTN_ERR_CUDA;
    }
    if (prop.major != 10 || prop.minor != 0) {
        fail(ctx, KD_ATTN_ERR_UNSUPPORTED, "device %d is sm_%d%d; libkd_attn is built for sm_100a only", ctx->device,
             prop.major, prop.minor);
        delete ctx;
        return KD_ATTN_ERR_UNSUPPORTED;
    }
    ctx->num_sms = prop.multiProcessorCount;
    if (cudaMalloc(&ctx->d_words, 8 * sizeof(unsigned)) != cudaSuccess ||
        cudaMemset(ctx->d_words, 0, 8 * sizeof(unsigned)) != cudaSuccess ||
        cudaMalloc(&ctx->d_barrier, 64) != cudaSuccess || cudaMemset(ctx->d_barrier, 0, 64) != cudaSuccess) {
        cudaGetLastError();
        if (ctx->d_words) cudaFree(ctx->d_words);
        if (ctx->d_barrier) cudaFree(ctx->d_barrier);
        delete ctx;
        return KD_ATTN_ERR_OUT_OF_MEMORY;
    }
    if (ctx->n_ranks > 1) {
        Nccl* n = nccl();
        if (!n || !init->nccl_unique_id) {
            fail(ctx, KD_ATTN_ERR_NCCL, "n_ranks > 1 needs NCCL and an nccl_unique_id");
            cudaFree(ctx->d_words);
            cudaFree(ctx->d_barrier);
            delete ctx;
            return KD_ATTN_ERR_NCCL;
        }
        NcclUid id;
        memcpy(id.internal, init->nccl_unique_id, sizeof id.internal);
        const int r = n->commInitRank(&ctx->nccl_comm, ctx->n_ranks, id, ctx->rank);
        if (r != 0) {
            fail(ctx, KD_ATTN_ERR_NCCL, "ncclCommInitRank: %s", nccl_err(n, r));
            cudaFree(ctx->d_words);
            cudaFree(ctx->d_barrier);
            delete ctx;
            return KD_ATTN_ERR_NCCL;
        }
    }
    *out = ctx;
    return KD_ATTN_OK;
}

void kd_attn_destroy(kd_attn_ctx* ctx) {
    if (!ctx) return;
    DeviceGuard g(ctx->device);
    if (ctx->h2d) {
        cudaStreamSynchronize(ctx->h2d);
        cudaStreamSynchronize(ctx->d2h);
        cudaStreamDestroy(ctx->h2d);
        cudaStreamDestroy(ctx->d2h);
        for (int i = 0; i < 2; ++i) {
            cudaEventDestroy(ctx->ev_in[i]);
            cudaEventDestroy(ctx->ev_done[i]);
            cudaEventDestroy(ctx->ev_out[i]);
        }
        cudaEventDestroy(ctx->ev_start);
        cudaEventDestroy(ctx->ev_last);
    }
    // Symmetric buffers: close this process's mappings of the peers' copies, free its own.  No
    // kernel of any rank may still be writing (callers destroy after their last step completed).
    for (auto& b : ctx->sym) release_sym(ctx, b);
    ctx->sym.clear();
    if (ctx->nccl_comm) {
        if (Nccl* n = nccl()) n->commDestroy(ctx->nccl_comm);
    }
    if (ctx->d_barrier) cudaFree(ctx->d_barrier);
    if (ctx->scratch) cudaFree(ctx->scratch);
    if (ctx->d_words) cudaFree(ctx->d_words);
    delete ctx;
}

const char* kd_attn_last_error(const kd_attn_ctx* ctx) { return ctx ? ctx->last_error.c_str() : ""; }

kd_attn_status kd_attn_device_status(kd_attn_ctx* ctx, void* stream) {
    if (!ctx) return KD_ATTN_ERR_INVALID_ARGUMENT;
    DeviceGuard g(ctx->device);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    KD_CUDA(ctx, cudaStreamSynchronize(st));
    unsigned words[2] = {0, 0};
    KD_CUDA(ctx, cudaMemcpy(words, ctx->d_words, sizeof words, cudaMemcpyDeviceToHost));
    KD_CUDA(ctx, cudaMemset(ctx->d_words, 0, sizeof words));
    if (words[0])
        return fail(ctx, KD_ATTN_ERR_DEVICE_TIMEOUT, "device-side wait expired (error bits 0x%x)", words[0]);
    return KD_ATTN_OK;
}

void kd_attn_set_log_callback(kd_attn_log_cb cb, void* user_data) {
    std::lock_guard<std::mutex> lock(g_log_mu);
    g_log_cb = cb;
    g_log_user = user_data;
}

kd_attn_status kd_attn_selftest_wait(kd_attn_ctx* ctx, uint32_t wait_ms, void* stream) {
    if (!ctx || wait_ms == 0 || wait_ms > 10000) return KD_ATTN_ERR_INVALID_ARGUMENT;
    DeviceGuard g(ctx->device);
    KD_CUDA(ctx, launch_wait_selftest(ctx->d_words, ctx->d_words + 1, (unsigned long long)wait_ms * 1000000ull,
                                      static_cast<cudaStream_t>(stream)));
    return KD_ATTN_OK;
}

kd_attn_status kd_attn_tile_stats(kd_attn_ctx* ctx, void* stream, uint64_t out[2], int32_t reset) {
    if (!ctx || !out) return KD_ATTN_ERR_INVALID_ARGUMENT;
    DeviceGuard g(ctx->device);
    KD_CUDA(ctx, cudaStreamSynchronize(static_cast<cudaStream_t>(stream)));
    unsigned long long v[2] = {0, 0};
    KD_CUDA(ctx, cudaMemcpy(v, ctx->d_words + 4, sizeof v, cudaMemcpyDeviceToHost));
    out[0] = v[0];
    out[1] = v[1];
    if (reset) KD_CUDA(ctx, cudaMemset(ctx->d_words + 4, 0, sizeof v));
    return KD_ATTN_OK;
}

kd_attn_status kd_attn_prologue(kd_attn_ctx* ctx, const kd_tensor* x, int32_t n_head, int32_t norm, const float* gain,
                                float eps, const kd_rope3d* rope, kd_tensor* y, void* stream) {
    if (!ctx) return KD_ATTN_ERR_INVALID_ARGUMENT;
    DeviceGuard g(ctx->device);
    return prologue_core(ctx, x, n_head, norm, gain, eps, rope, y, static_cast<cudaStream_t>(stream));
}

kd_attn_status kd_attn_qk_prologue(kd_attn_ctx* ctx, const kd_tensor* q_in, const kd_tensor* k_in,
                                   const kd_tensor* v_in, const float* q_gain, const float* k_gain, float eps,
                                   const kd_rope3d* rope, int32_t out_dtype, kd_tensor* q_out, kd_tensor* k_out,
                                   kd_tensor* v_out, void* stream) {
    if (!ctx) return KD_ATTN_ERR_INVALID_ARGUMENT;
    DeviceGuard g(ctx->device);
    const kd_tensor* ins[3] = {q_in, k_in, v_in};
    kd_tensor* outs[3] = {q_out, k_out, v_out};
    PrologueReq req[3];
    int count = 0;
    int64_t n_head = -1;
    for (int i = 0; i < 3; ++i) {
        if (!ins[i] && !outs[i]) continue;
        if (!ins[i] || !outs[i]) return fail(ctx, KD_ATTN_ERR_INVALID_ARGUMENT, "input and output must both be given");
        if (outs[i]->type != out_dtype)
            return fail(ctx, KD_ATTN_ERR_INVALID_ARGUMENT, "outputs must have type out_dtype");
        if (n_head >= 0 && outs[i]->ne[2] != n_head)
            return fail(ctx, KD_ATTN_ERR_INVALID_ARGUMENT, "outputs disagree on the head count");
        n_head = outs[i]->ne[2];
        req[count++] = PrologueReq{ins[i], i < 2 ? 1 : 0, i == 0 ? q_gain : (i == 1 ? k_gain : nullptr), i < 2, outs[i]};
    }
    if (count == 0) return KD_ATTN_OK;
    if (out_dtype != KD_ATTN_TYPE_F32 && out_dtype != KD_ATTN_TYPE_F16 && out_dtype != KD_ATTN_TYPE_BF16)
        return fail(ctx, KD_ATTN_ERR_UNSUPPORTED, "out_dtype must be f32, f16 or bf16");
    if (n_head <= 0 || n_head > (1 << 20)) return fail(ctx, KD_ATTN_ERR_INVALID_ARGUMENT, "bad head count");
    return prologue_multi(ctx, req, count, (int32_t)n_head, eps, rope, static_cast<cudaStream_t>(stream));
}

kd_attn_status kd_attn_qkv_projection(kd_attn_ctx* ctx, const kd_tensor* x, const kd_linear* wq, const kd_linear* wk,
                                      const kd_linear* wv, const float* q_gain, const float* k_gain, float eps,
                                      const kd_rope3d* rope, int32_t out_dtype, kd_tensor* q_out, kd_tensor* k_out,
                                      kd_tensor* v_out, void* stream) {
    if (!ctx) return KD_ATTN_ERR_INVALID_ARGUMENT;
    DeviceGuard g(ctx->device);
    const kd_linear* w[3] = {wq, wk, wv};
    kd_tensor* outs[3] = {q_out, k_out, v_out};
    return qkv_projection_core(ctx, x, w, q_gain, k_gain, eps, rope, out_dtype, outs, static_cast<cudaStream_t>(stream));
}

kd_attn_status kd_attn_linear(kd_attn_ctx* ctx, const kd_tensor* x, const kd_linear* w, kd_tensor* y, void* stream) {
    if (!ctx) return KD_ATTN_ERR_INVALID_ARGUMENT;
    DeviceGuard g(ctx->device);
    return linear_core(ctx, x, w, y, static_cast<cudaStream_t>(stream));
}

kd_attn_status kd_attn_self_attention_block(kd_attn_ctx* ctx, const kd_tensor* x, const kd_linear* wq,
                                            const kd_linear* wk, const kd_linear* wv, const kd_linear* wo,
                                            int32_t n_head, const float* q_gain, const float* k_gain, float eps,
                                            const kd_rope3d* rope, kd_tensor* y, void* stream) {
    if (!ctx) return KD_ATTN_ERR_INVALID_ARGUMENT;
    DeviceGuard g(ctx->device);
    return self_attention_block_core(ctx, x, wq, wk, wv, wo, n_head, q_gain, k_gain, eps, rope, y,
                                     static_cast<cudaStream_t>(stream));
}

kd_attn_status kd_attn_cross_attention_block(kd_attn_ctx* ctx, const kd_tensor* x_query, const kd_tensor* x_kv,
                                             const kd_linear* wq, const kd_linear* wk, const kd_linear* wv,
                                             const kd_linear* wo, int32_t n_head, const float* q_gain,
                                             const float* k_gain, float eps, const kd_tensor* mask,
                                             const int32_t* kv_len, kd_tensor* y, void* stream) {
    if (!ctx) return KD_ATTN_ERR_INVALID_ARGUMENT;
    DeviceGuard g(ctx->device);
    return cross_attention_block_core(ctx, x_query, x_kv, wq, wk, wv, wo, n_head, q_gain, k_gain, eps, mask, kv_len,
                                      y, static_cast<cudaStream_t>(stream));
}

kd_attn_status kd_attn_flash_ext(kd_attn_ctx* ctx, const kd_tensor* q, const kd_tensor* k, const kd_tensor* v,
                                 const kd_tensor* mask, float scale, float max_bias, float logit_softcap,
                                 const int32_t* kv_len, const uint8_t* tile_mask, kd_tensor* out, float* lse,
                                 void* stream) {
    if (!ctx) return KD_ATTN_ERR_INVALID_ARGUMENT;
    if (max_bias != 0.f) return fail(ctx, KD_ATTN_ERR_UNSUPPORTED, "max_bias (ALiBi) must be 0");
    if (logit_softcap != 0.f) return fail(ctx, KD_ATTN_ERR_UNSUPPORTED, "logit_softcap must be 0");
    DeviceGuard g(ctx->device);
    FlashArgs fa{q, k, v, mask, scale, kv_len, out, lse, tile_mask};
    return flash_run(ctx, fa, static_cast<cudaStream_t>(stream));
}

kd_attn_status kd_attn_self_attention(kd_attn_ctx* ctx, const kd_tensor* q_in, const kd_tensor* k_in,
                                      const kd_tensor* v_in, int32_t n_head, const float* q_gain, const float* k_gain,
                                      float eps, const kd_rope3d* rope, int32_t op_type, kd_tensor* out, float* lse,
                                      void* stream) {
    if (!ctx) return KD_ATTN_ERR_INVALID_ARGUMENT;
    DeviceGuard g(ctx->device);
    if (q_in && k_in && q_in->ne[1] != k_in->ne[1])
        return fail(ctx, KD_ATTN_ERR_INVALID_ARGUMENT, "self-attention needs Lq == Lk");
    return attention_core(ctx, q_in, k_in, v_in, n_head, q_gain, k_gain, eps, rope, nullptr, nullptr, op_type, out, lse,
                          static_cast<cudaStream_t>(stream));
}

kd_attn_status kd_attn_self_attention_host(kd_attn_ctx* ctx, const kd_tensor* q_in, const kd_tensor* k_in,
                                           const kd_tensor* v_in, int32_t n_head, const float* q_gain,
                                           const float* k_gain, float eps, const kd_rope3d* rope, int32_t op_type,
                                           kd_tensor* out, void* stream) {
    if (!ctx) return KD_ATTN_ERR_INVALID_ARGUMENT;
    DeviceGuard g(ctx->device);
    return self_attention_host(ctx, q_in, k_in, v_in, n_head, q_gain, k_gain, eps, rope, op_type, out,
                               static_cast<cudaStream_t>(stream));
}

kd_attn_status kd_attn_attention(kd_attn_ctx* ctx, const kd_tensor* q_in, const kd_tensor* k_in, const kd_tensor* v_in,
                                 int32_t n_head, const kd_tensor* mask, int32_t op_type, kd_tensor* out, float* lse,
                                 void* stream) {
    if (!ctx) return KD_ATTN_ERR_INVALID_ARGUMENT;
    DeviceGuard g(ctx->device);
    return attention_core(ctx, q_in, k_in, v_in, n_head, nullptr, nullptr, 0.f, nullptr, mask, nullptr, op_type, out,
                          lse, static_cast<cudaStream_t>(stream), nullptr, nullptr, 0, /*norm_qk=*/false);
}

kd_attn_status kd_attn_cross_attention(kd_attn_ctx* ctx, const kd_tensor* q_in, const kd_tensor* k_in,
                                       const kd_tensor* v_in, int32_t n_head, const float* q_gain, const float* k_gain,
                                       float eps, const kd_tensor* mask, const int32_t* kv_len, int32_t op_type,
                                       kd_tensor* out, float* lse, void* stream) {
    if (!ctx) return KD_ATTN_ERR_INVALID_ARGUMENT;
    DeviceGuard g(ctx->device);
    return attention_core(ctx, q_in, k_in, v_in, n_head, q_gain, k_gain, eps, nullptr, mask, kv_len, op_type, out, lse,
                          static_cast<cudaStream_t>(stream));
}

kd_attn_status kd_attn_symmetric_alloc(kd_attn_ctx* ctx, size_t bytes, void** out) {
    if (!ctx || !out || bytes == 0) return KD_ATTN_ERR_INVALID_ARGUMENT;
    *out = nullptr;
    DeviceGuard g(ctx->device);
    const int R = ctx->n_ranks;
    if (R > 8) return fail(ctx, KD_ATTN_ERR_UNSUPPORTED, "symmetric buffers span at most 8 ranks");
    kd_attn_ctx::SymBuf b;
    b.bytes = align256(bytes);
    if (cudaMalloc(reinterpret_cast<void**>(&b.local), b.bytes) != cudaSuccess) {
        cudaGetLastError();
        return fail(ctx, KD_ATTN_ERR_OUT_OF_MEMORY, "could not allocate %zu bytes", b.bytes);
    }
    b.peer[ctx->rank] = b.local;
    if (R > 1) {
        Nccl* n = nccl();
        if (!n || !ctx->nccl_comm) {
            cudaFree(b.local);
            return fail(ctx, KD_ATTN_ERR_NCCL, "context has no NCCL communicator");
        }
        // exchange IPC handles: one 64-byte handle per rank, all-gathered over the communicator
        cudaIpcMemHandle_t mine;
        std::vector<cudaIpcMemHandle_t> all(R);
        unsigned char* dev = nullptr;
        cudaStream_t s = nullptr;
        kd_attn_status rc = KD_ATTN_OK;
        cudaError_t e = cudaIpcGetMemHandle(&mine, b.local);
        if (e == cudaSuccess) e = cudaMalloc(&dev, sizeof(cudaIpcMemHandle_t) * (R + 1));
        if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking);
        if (e == cudaSuccess) e = cudaMemcpyAsync(dev, &mine, sizeof mine, cudaMemcpyHostToDevice, s);
        if (e == cudaSuccess) {
            const int r = n->allGather(dev, dev + sizeof mine, sizeof mine, kNcclUint8, ctx->nccl_comm, s);
            if (r != 0) rc = fail(ctx, KD_ATTN_ERR_NCCL, "ncclAllGather (IPC handles): %s", nccl_err(n, r));
        }
        if (e == cudaSuccess && rc == KD_ATTN_OK)
            e = cudaMemcpyAsync(all.data(), dev + sizeof mine, sizeof mine * R, cudaMemcpyDeviceToHost, s);
        if (e == cudaSuccess && rc == KD_ATTN_OK) e = cudaStreamSynchronize(s);
        for (int i = 0; e == cudaSuccess && rc == KD_ATTN_OK && i < R; ++i)
            if (i != ctx->rank)
                e = cudaIpcOpenMemHandle(reinterpret_cast<void**>(&b.peer[i]), all[i], cudaIpcMemLazyEnablePeerAccess);
        if (s) cudaStreamDestroy(s);
        if (dev) cudaFree(dev);
        if (e != cudaSuccess && rc == KD_ATTN_OK)
            rc = fail(ctx, KD_ATTN_ERR_CUDA, "symmetric buffer setup failed: %s", cudaGetErrorString(e));
        if (rc != KD_ATTN_OK) {
            cudaGetLastError();
            release_sym(ctx, b);
            return rc;
        }
    }
    ctx->sym.push_back(b);
    *out = b.local;
    return KD_ATTN_OK;
}

kd_attn_status kd_attn_symmetric_free(kd_attn_ctx* ctx, void* ptr, void* stream) {
    if (!ctx || !ptr) return KD_ATTN_ERR_INVALID_ARGUMENT;
    DeviceGuard g(ctx->device);
    for (size_t i = 0; i < ctx->sym.size(); ++i) {
        if (ctx->sym[i].local != ptr) continue;
        cudaStream_t st = static_cast<cudaStream_t>(stream);
        kd_attn_status rc;
        // no rank may still be writing into any copy
        if ((rc = rank_barrier(ctx, st))) return rc;
        KD_CUDA(ctx, cudaStreamSynchronize(st));
        release_sym(ctx, ctx->sym[i]);
        ctx->sym.erase(ctx->sym.begin() + (long)i);
        return KD_ATTN_OK;
    }
    return fail(ctx, KD_ATTN_ERR_INVALID_ARGUMENT, "not a symmetric buffer of this context");
}

}  // extern "C"

namespace {

// Head-sharded attention into a symmetric out_full: barrier, this rank's heads (prologue + flash whose
// copy-out warp also stores every row into the other ranks' copies), barrier.
kd_attn_status sharded_core(kd_attn_ctx* ctx, const kd_tensor* q_in, const kd_tensor* k_in, const kd_tensor* v_in,
                            int32_t n_head_local, const float* q_gain, const float* k_gain, float eps,
                            const kd_rope3d* rope, const kd_tensor* mask, const int32_t* kv_len, int32_t op_type,
                            kd_tensor* out_full, cudaStream_t st) {
    kd_attn_status rc;
    if ((rc = check_tensor(ctx, out_full, "out_full")) || (rc = check_tensor(ctx, q_in, "q_in"))) return rc;
    const int R = ctx->n_ranks;
    // head dim D = q_in.ne[0] / n_head_local (128, or 64; attention_core checks it)
    const int64_t D = n_head_local > 0 ? q_in->ne[0] / n_head_local : 0;
    const int64_t C = (int64_t)n_head_local * R * D;
    if (n_head_local <= 0 || out_full->ne[0] != C || out_full->ne[3] != 1)
        return fail(ctx, KD_ATTN_ERR_INVALID_ARGUMENT, "out_full must be [n_head_local * n_ranks * D, L, N]");
    const size_t es = elt_size(out_full->type);
    if (out_full->nb[0] != es || out_full->nb[2] < out_full->nb[1] * (size_t)out_full->ne[1])
        return fail(ctx, KD_ATTN_ERR_UNSUPPORTED, "out_full rows must be contiguous and sequences not overlapping");
    const size_t extent = out_full->nb[2] * (size_t)(out_full->ne[2] - 1) + out_full->nb[1] * (size_t)(out_full->ne[1] - 1) +
                          (size_t)C * es;
    char* peers[kMaxPeers];
    int np = 0;
    const char* base = nullptr;
    if (R > 1) {
        kd_attn_ctx::SymBuf* b = find_sym(ctx, out_full->data, out_full->ne[1] * out_full->ne[2] ? extent : 0);
        if (!b) return fail(ctx, KD_ATTN_ERR_INVALID_ARGUMENT, "out_full must lie in a kd_attn_symmetric_alloc buffer");
        for (int i = 0; i < R; ++i)
            if (i != ctx->rank) peers[np++] = b->peer[i];
        base = b->local;
    }
    // this rank's heads are columns [rank * n_head_local * D, +n_head_local * D) of every copy
    kd_tensor cols = *out_full;
    cols.data = static_cast<char*>(out_full->data) + (size_t)ctx->rank * n_head_local * D * es;
    cols.ne[0] = (int64_t)n_head_local * D;
    if ((rc = rank_barrier(ctx, st))) return rc;  // nobody still reads the previous contents
    if ((rc = attention_core(ctx, q_in, k_in, v_in, n_head_local, q_gain, k_gain, eps, rope, mask, kv_len, op_type,
                             &cols, nullptr, st, base, peers, np)))
        return rc;
    return rank_barrier(ctx, st);  // every rank's rows have landed in every copy
}

// DiTSelfAttention::forward with heads sharded over the group: this rank's column shard of the Q/K/V
// weights (its n_head_local heads) projects the replicated hidden states x, the flash kernel's epilogue
// stores this rank's heads into every rank's attn_full (the fused exchange), and after the closing
// barrier every rank runs the out-projection on the gathered attention output -- the all-gather ->
// out_layer order of crossdit.hpp:150-153.  Scratch: [Q][K][V operands][GEMM work].
kd_attn_status self_attention_block_sharded_core(kd_attn_ctx* ctx, const kd_tensor* x, const kd_linear* wq,
                                                 const kd_linear* wk, const kd_linear* wv, const kd_linear* wo,
                                                 int32_t n_head_local, const float* q_gain, const float* k_gain,
                                                 float eps, const kd_rope3d* rope, kd_tensor* attn_full,
                                                 kd_tensor* y, cudaStream_t st) {
    kd_attn_status rc;
    GemmInput in;
    if ((rc = gemm_input(ctx, x, &in))) return rc;
    if (!wq || !wk || !wv || !wo) return fail(ctx, KD_ATTN_ERR_INVALID_ARGUMENT, "all four weights are required");
    if ((rc = check_tensor(ctx, attn_full, "attn_full"))) return rc;
    const int R = ctx->n_ranks;
    const int64_t Cl = wq->ne[1], C = Cl * R, L = in.L, N = in.N;
    if (wk->ne[1] != Cl || wv->ne[1] != Cl || wo->ne[0] != C)
        return fail(ctx, KD_ATTN_ERR_INVALID_ARGUMENT,
                    "wq/wk/wv must be this rank's n_head_local * D output features and wo take all n_ranks of them");
    const int64_t D = n_head_local > 0 ? Cl / n_head_local : 0;
    if (n_head_local <= 0 || (D != kHeadDim && D != kHeadDim64) || (int64_t)n_head_local * D != Cl)
        return fail(ctx, KD_ATTN_ERR_UNSUPPORTED, "C_local = %lld over %d heads is not a head dim of 128 or 64",
                    (long long)Cl, n_head_local);
    if (attn_full->type != KD_ATTN_TYPE_BF16 || attn_full->ne[0] != C || attn_full->ne[1] != L ||
        attn_full->ne[2] != N || attn_full->ne[3] != 1 || attn_full->nb[0] != 2 ||
        attn_full->nb[1] != 2 * (size_t)C || attn_full->nb[2] != attn_full->nb[1] * (size_t)L)
        return fail(ctx, KD_ATTN_ERR_INVALID_ARGUMENT, "attn_full must be a contiguous bf16 [n_ranks * C_local, L, N]");
    const int32_t Hl = n_head_local;
    const int32_t op = KD_ATTN_TYPE_BF16;
    const size_t opb = align256((size_t)N * Hl * L * D * 2);
    const bool rot = rope != nullptr;
    GemmInput attn_in = in;  // the out-projection reads attn_full in place
    attn_in.x = attn_full;
    attn_in.K = attn_in.Kp = C;
    attn_in.direct = true;
    const size_t work = std::max(gemm_work_bytes(in, 3, Cl, rot), gemm_work_bytes(attn_in, 1, wo->ne[1], false));
    if ((rc = ensure_scratch(ctx, 3 * opb + work, st))) return rc;
    char* base = static_cast<char*>(ctx->scratch);
    kd_tensor Qs = operand_view(base, op, L, Hl, N, D);
    kd_tensor Ks = operand_view(base + opb, op, L, Hl, N, D);
    kd_tensor Vs = operand_view(base + 2 * opb, op, L, Hl, N, D);
    char* gw = base + 3 * opb;
    const kd_linear* w3[3] = {wq, wk, wv};
    kd_tensor* o3[3] = {&Qs, &Ks, &Vs};
    if ((rc = qkv_projection_core(ctx, x, w3, q_gain, k_gain, eps, rope, op, o3, st, gw))) return rc;
    const size_t extent = attn_full->nb[2] * (size_t)N;
    char* peers[kMaxPeers];
    int np = 0;
    const char* sbase = nullptr;
    if (R > 1) {
        kd_attn_ctx::SymBuf* b = find_sym(ctx, attn_full->data, L * N ? extent : 0);
        if (!b) return fail(ctx, KD_ATTN_ERR_INVALID_ARGUMENT, "attn_full must lie in a kd_attn_symmetric_alloc buffer");
        for (int i = 0; i < R; ++i)
            if (i != ctx->rank) peers[np++] = b->peer[i];
        sbase = b->local;
    }
    kd_tensor cols = *attn_full;  // this rank's heads: columns [rank * Cl, (rank + 1) * Cl) of every copy
    cols.data = static_cast<char*>(attn_full->data) + (size_t)ctx->rank * Cl * 2;
    cols.ne[0] = Cl;
    kd_tensor ov;
    if ((rc = out_view(ctx, &cols, Hl, L, N, &ov, D))) return rc;
    if ((rc = rank_barrier(ctx, st))) return rc;  // nobody still reads the previous contents of its copy
    FlashArgs fa{&Qs, &Ks, &Vs, nullptr, 1.0f / std::sqrt((float)D), nullptr, &ov, nullptr};
    fa.out_base = sbase;
    fa.peer_base = peers;
    fa.n_peers = np;
    if ((rc = flash_run(ctx, fa, st))) return rc;
    if ((rc = rank_barrier(ctx, st))) return rc;  // every rank's heads have landed in every copy
    // The out-projection.  y in a symmetric buffer (contiguous rows): rank r computes token rows
    // [r*M/R, (r+1)*M/R) of y = out_layer(attn_full), the copy engines put that block into every other
    // rank's copy, and a barrier closes the call; otherwise every rank computes all rows.  (Storing the
    // rows to the peers from the GEMM epilogue -- 16 bytes per lane to 32 rows per instruction -- made the
    // 2-GPU block slower than computing every row on every rank: 20.3 vs 19.2 ms.)
    if ((rc = check_tensor(ctx, y, "y"))) return rc;
    const size_t ye = elt_size(y->type);
    const int64_t Co = wo->ne[1], M = L * N;
    kd_attn_ctx::SymBuf* yb = nullptr;
    if (R > 1 && y->ne[0] == Co && y->ne[1] == L && y->ne[2] == N && y->ne[3] == 1 && y->nb[0] == ye &&
        y->nb[1] == (size_t)Co * ye && y->nb[2] == y->nb[1] * (size_t)L && M > 0)
        yb = find_sym(ctx, y->data, y->nb[1] * (size_t)M);
    if (!yb) return linear_core(ctx, attn_full, wo, y, st, gw);
    const int64_t m0 = M * ctx->rank / R, m1 = M * (ctx->rank + 1) / R;
    kd_tensor xs = *attn_full, ys = *y;  // [C, M, 1] and [C_out, M, 1] views, rows [m0, m1)
    xs.data = static_cast<char*>(attn_full->data) + (size_t)m0 * attn_full->nb[1];
    ys.data = static_cast<char*>(y->data) + (size_t)m0 * y->nb[1];
    xs.ne[1] = ys.ne[1] = m1 - m0;
    xs.ne[2] = ys.ne[2] = 1;
    xs.nb[2] = xs.nb[3] = attn_full->nb[1] * (size_t)(m1 - m0);
    ys.nb[2] = ys.nb[3] = y->nb[1] * (size_t)(m1 - m0);
    if (m1 > m0) {
        if ((rc = linear_core(ctx, &xs, wo, &ys, st, gw))) return rc;
        // this rank's rows, one contiguous block, into every other rank's copy by the copy engines
        const size_t off = static_cast<char*>(ys.data) - yb->local, bytes = y->nb[1] * (size_t)(m1 - m0);
        for (int i = 0; i < R; ++i)
            if (i != ctx->rank)
                KD_CUDA(ctx, cudaMemcpyAsync(yb->peer[i] + off, ys.data, bytes, cudaMemcpyDeviceToDevice, st));
    }
    return rank_barrier(ctx, st);  // every rank's rows of y have landed in every copy
}

}  // namespace

extern "C" {

kd_attn_status kd_attn_self_attention_block_sharded(kd_attn_ctx* ctx, const kd_tensor* x, const kd_linear* wq,
                                                    const kd_linear* wk, const kd_linear* wv, const kd_linear* wo,
                                                    int32_t n_head_local, const float* q_gain, const float* k_gain,
                                                    float eps, const kd_rope3d* rope, kd_tensor* attn_full,
                                                    kd_tensor* y, void* stream) {
    if (!ctx) return KD_ATTN_ERR_INVALID_ARGUMENT;
    DeviceGuard g(ctx->device);
    return self_attention_block_sharded_core(ctx, x, wq, wk, wv, wo, n_head_local, q_gain, k_gain, eps, rope,
                                             attn_full, y, static_cast<cudaStream_t>(stream));
}

kd_attn_status kd_attn_self_attention_sharded(kd_attn_ctx* ctx, const kd_tensor* q_in, const kd_tensor* k_in,
                                              const kd_tensor* v_in, int32_t n_head_local, const float* q_gain,
                                              const float* k_gain, float eps, const kd_rope3d* rope,
                                              int32_t op_type, kd_tensor* out_full, void* stream) {
    if (!ctx) return KD_ATTN_ERR_INVALID_ARGUMENT;
    DeviceGuard g(ctx->device);
    return sharded_core(ctx, q_in, k_in, v_in, n_head_local, q_gain, k_gain, eps, rope, nullptr, nullptr, op_type,
                        out_full, static_cast<cudaStream_t>(stream));
}

kd_attn_status kd_attn_cross_attention_sharded(kd_attn_ctx* ctx, const kd_tensor* q_in, const kd_tensor* k_in,
                                               const kd_tensor* v_in, int32_t n_head_local, const float* q_gain,
                                               const float* k_gain, float eps, const kd_tensor* mask,
                                               const int32_t* kv_len, int32_t op_type, kd_tensor* out_full,
                                               void* stream) {
    if (!ctx) return KD_ATTN_ERR_INVALID_ARGUMENT;
    DeviceGuard g(ctx->device);
    return sharded_core(ctx, q_in, k_in, v_in, n_head_local, q_gain, k_gain, eps, nullptr, mask, kv_len, op_type,
                        out_full, static_cast<cudaStream_t>(stream));
}

kd_attn_status kd_attn_allgather_heads(kd_attn_ctx* ctx, const kd_tensor* shard, kd_tensor* full, void* stream) {
    if (!ctx) return KD_ATTN_ERR_INVALID_ARGUMENT;
    kd_attn_status rc;
    if ((rc = check_tensor(ctx, shard, "shard")) || (rc = check_tensor(ctx, full, "full"))) return rc;
    if (shard->type != full->type) return fail(ctx, KD_ATTN_ERR_INVALID_ARGUMENT, "shard and full types differ");
    const int R = ctx->n_ranks;
    const int64_t D = shard->ne[0], Hs = shard->ne[1], Lq = shard->ne[2], N = shard->ne[3];
    if (full->ne[0] != D || full->ne[1] != Hs * R || full->ne[2] != Lq || full->ne[3] != N)
        return fail(ctx, KD_ATTN_ERR_INVALID_ARGUMENT, "full must be [D, H_shard * n_ranks, Lq, N]");
    const size_t es = elt_size(shard->type);
    const size_t row = (size_t)D * Hs * es;
    auto contiguous = [&](const kd_tensor* t, int64_t heads) {
        return t->nb[1] == (size_t)D * es && t->nb[2] == (size_t)D * heads * es &&
               t->nb[3] == (size_t)D * heads * Lq * es;
    };
    if (!contiguous(shard, Hs) || !contiguous(full, Hs * R) || row % 16 || !aligned16(full->data))
        return fail(ctx, KD_ATTN_ERR_UNSUPPORTED, "allgather_heads needs contiguous, 16-byte aligned rows");
    const size_t shard_bytes = row * (size_t)Lq * N;
    if (shard_bytes == 0) return KD_ATTN_OK;
    DeviceGuard g(ctx->device);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (R == 1) {
        KD_CUDA(ctx, cudaMemcpyAsync(full->data, shard->data, shard_bytes, cudaMemcpyDeviceToDevice, st));
        return KD_ATTN_OK;
    }
    Nccl* n = nccl();
    if (!n || !ctx->nccl_comm) return fail(ctx, KD_ATTN_ERR_NCCL, "context has no NCCL communicator");
    if ((rc = ensure_scratch(ctx, shard_bytes * R, st))) return rc;
    const int r = n->allGather(shard->data, ctx->scratch, shard_bytes, kNcclUint8, ctx->nccl_comm, st);
    if (r != 0) return fail(ctx, KD_ATTN_ERR_NCCL, "ncclAllGather: %s", nccl_err(n, r));
    KD_CUDA(ctx, launch_unshard_heads(ctx->scratch, full->data, (long long)Lq * N, R, (long long)row, ctx->num_sms, st));
    return KD_ATTN_OK;
}

kd_attn_status kd_attn_fill_randn(kd_attn_ctx* ctx, float* dst, uint64_t n, uint64_t seed, uint32_t offset,
                                  void* stream) {
    if (!ctx || (n && !dst)) return KD_ATTN_ERR_INVALID_ARGUMENT;
    if (n > 0xffffffffull) return fail(ctx, KD_ATTN_ERR_UNSUPPORTED, "randn counter index is 32-bit (n <= 2^32)");
    DeviceGuard g(ctx->device);
    KD_CUDA(ctx, launch_randn(dst, n, seed, offset, ctx->num_sms, static_cast<cudaStream_t>(stream)));
    return KD_ATTN_OK;
}

}  // extern "C"

// ====================================================================== allocation-free flash entry
extern "C" kd_attn_status kd_attn_flash_ext_noalloc(const kd_tensor* q, const kd_tensor* k, const kd_tensor* v,
                                                    const kd_tensor* mask, float scale, float max_bias,
                                                    float logit_softcap, const int32_t* kv_len,
                                                    const uint8_t* tile_mask, kd_tensor* out, float* lse,
                                                    void* stream) {
    if (max_bias != 0.f) return fail(nullptr, KD_ATTN_ERR_UNSUPPORTED, "max_bias (ALiBi) must be 0");
    if (logit_softcap != 0.f) return fail(nullptr, KD_ATTN_ERR_UNSUPPORTED, "logit_softcap must be 0");
    FlashArgs fa{q, k, v, mask, scale, kv_len, out, lse, tile_mask};
    return flash_run(nullptr, fa, static_cast<cudaStream_t>(stream));
}

extern "C" kd_attn_status kd_attn_noalloc_status(void* stream) {
    NoAllocDevice* d = nullptr;
    kd_attn_status rc;
    if ((rc = noalloc_setup(&d))) return rc;
    cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
    unsigned word = 0;
    if (e == cudaSuccess) e = cudaMemcpy(&word, d->words, sizeof word, cudaMemcpyDeviceToHost);
    if (e == cudaSuccess) e = cudaMemset(d->words, 0, sizeof word);
    if (e != cudaSuccess) return fail(nullptr, KD_ATTN_ERR_CUDA, "reading the allocation-free error word: %s",
                                      cudaGetErrorString(e));
    if (word)
        return fail(nullptr, KD_ATTN_ERR_DEVICE_TIMEOUT, "device-side wait expired in the allocation-free path "
                    "(error bits 0x%x)", word);
    return KD_ATTN_OK;
}

extern "C" kd_attn_status kd_attn_noalloc_selftest_wait(uint32_t wait_ms, void* stream) {
    if (wait_ms == 0 || wait_ms > 10000) return KD_ATTN_ERR_INVALID_ARGUMENT;
    NoAllocDevice* d = nullptr;
    kd_attn_status rc;
    if ((rc = noalloc_setup(&d))) return rc;
    const cudaError_t e = launch_wait_selftest(d->words, d->words + 1, (unsigned long long)wait_ms * 1000000ull,
                                               static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return fail(nullptr, KD_ATTN_ERR_CUDA, "self-test launch: %s", cudaGetErrorString(e));
    return KD_ATTN_OK;
}
