// C ABI for CQ matrices on B200: handle lifetime, host validation, staging
// and the error channel.  Mirrors the reference entry points of
// needle2/csrc/cq.cpp:342-371 and needle2/csrc/sdot.cpp:349-360; all
// arithmetic runs in the kernels of cq_kernels.cu.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <mutex>
#include <new>
#include <string>
#include <vector>

#include "../../include/needle2_b200.h"
#include "common.cuh"
#include "cq_gemv.cuh"
#include "cq_handle.cuh"
#include "cq_kernels.cuh"

namespace nb200 {

static thread_local std::string g_error;
void set_error(const std::string &msg) { g_error = msg; }
void clear_error() { g_error.clear(); }
const char *last_error() { return g_error.c_str(); }

namespace {

// Device buffer that only grows.
template <typename T>
struct Scratch {
    T *ptr = nullptr;
    size_t cap = 0;
    bool reserve(size_t n) {
        if (n <= cap) return true;
        if (ptr) cudaFree(ptr);
        ptr = nullptr;
        cap = 0;
        cudaError_t e = cudaMalloc(&ptr, sizeof(T) * (n ? n : 1));
        if (e != cudaSuccess) {
            set_error(std::string("device scratch allocation failed: ") + cudaGetErrorString(e));
            ptr = nullptr;
            return false;
        }
        cap = n;
        return true;
    }
    void release() {
        if (ptr) cudaFree(ptr);
        ptr = nullptr;
        cap = 0;
    }
};

// Page-locked host staging for copies to or from pageable user buffers: one
// transfer of the whole batch instead of one staged transfer per matrix.
struct PinnedStage {
    float *ptr = nullptr;
    size_t cap = 0;
    bool reserve(size_t n) {
        if (n <= cap) return true;
        if (ptr) cudaFreeHost(ptr);
        ptr = nullptr;
        cap = 0;
        cudaError_t e = cudaMallocHost(&ptr, sizeof(float) * (n ? n : 1));
        if (e != cudaSuccess) {
            set_error(std::string("pinned staging allocation failed: ") + cudaGetErrorString(e));
            ptr = nullptr;
            return false;
        }
        cap = n;
        return true;
    }
    void release() {
        if (ptr) cudaFreeHost(ptr);
        ptr = nullptr;
        cap = 0;
    }
};

// True when p is page-locked (or device/managed) memory that async copies use directly.
inline bool is_pinned(const void *p) {
    cudaPointerAttributes a{};
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();   // an unregistered pointer may report an error on older drivers
        return false;
    }
    return a.type == cudaMemoryTypeHost || a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged;
}

// The device's address of page-locked host memory (kernels may store to it
// directly), or null when p is not page-locked host memory.
inline float *mapped_host(float *p) {
    cudaPointerAttributes a{};
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    return a.type == cudaMemoryTypeHost ? static_cast<float *>(a.devicePointer) : nullptr;
}

struct Matrix {
    CQDevice w{};
    bool sdot = false;
    int device = 0;
    cudaStream_t stream = nullptr;
    uint8_t *d_packed = nullptr;
    uint16_t *d_norms = nullptr;
    uint16_t *d_norms8 = nullptr;   // padded copy when groups % 8 != 0 (int8 mode)
    uint8_t *d_frag = nullptr;      // int8 mode: fragment-order weights for the warp-MMA kernel
    int8_t *d_w8 = nullptr;         // int8 mode: decoded weights for the prefill GEMM (made at first use)
    float *d_nsT = nullptr;         // int8 mode: group scales for the prefill GEMM
    uint16_t *d_whl = nullptr;      // FP32 mode: bf16 hi/lo weights for the prefill GEMM (made at first use)
    uint16_t *d_normsF = nullptr;   // int8 mode: fragment-order norms
    uint8_t *d_blocked = nullptr;   // FP32 mode: row-block weights for the decode GEMV
    uint16_t *d_normsB = nullptr;   // FP32 mode: row-block norms
    Scratch<float> x, y, rot, xs;
    Scratch<int8_t> q;
    Scratch<uint16_t> ahl;   // FP32 mode: bf16 hi/lo activations for the prefill GEMM
    PinnedStage hin, hout;   // host staging for pageable inputs / outputs of the host-pointer calls
    Scratch<int32_t> partials;
    Scratch<int64_t> ids;
    int prepared = 0;  // activation rows held in rot / q+xs by the last prepare

    ~Matrix() {
        cudaSetDevice(device);
        if (stream) cudaStreamSynchronize(stream);
        x.release(); y.release(); rot.release(); xs.release(); q.release(); partials.release(); ids.release();
        ahl.release(); hin.release(); hout.release();
        if (d_packed) cudaFree(d_packed);
        if (d_norms) cudaFree(d_norms);
        if (d_norms8) cudaFree(d_norms8);
        if (d_frag) cudaFree(d_frag);
        if (d_w8) cudaFree(d_w8);
        if (d_nsT) cudaFree(d_nsT);
        if (d_whl) cudaFree(d_whl);
        if (d_normsF) cudaFree(d_normsF);
        if (d_blocked) cudaFree(d_blocked);
        if (d_normsB) cudaFree(d_normsB);
        if (stream) cudaStreamDestroy(stream);
    }
};

bool is_pow2(int v) { return v > 0 && (v & (v - 1)) == 0; }

Matrix *create_matrix(const uint8_t *packed, const uint16_t *norms, int out, int in, int bits, int group,
                      const float *cb, bool sdot) {
    clear_error();
    if (!packed || !norms || !cb) { set_error("null packed/norms/codebook pointer"); return nullptr; }
    if (out <= 0 || in <= 0) { set_error("CQ requires a positive two-dimensional shape"); return nullptr; }
    if (bits != 2 && bits != 3 && bits != 4 && bits != 5) { set_error("CQ storage bits must be 2, 3, 4 or 5"); return nullptr; }
    if (!is_pow2(group) || group < 8) { set_error("CQ group size must be a power of two >= 8"); return nullptr; }
    if (group > kMaxGroup) { set_error("group size above 16384 is not supported by the GPU build"); return nullptr; }
    if (sdot && ((bits != 2 && bits != 4) || group < 64)) {
        set_error("SDOT requires CQ2/CQ4 and group size between 64 and 131072");
        return nullptr;
    }
    const long long padded = ((long long)in + group - 1) / group * group;
    const int sbits = bits == 5 ? 2 : bits;
    if (padded * sbits > 0x7fffffffLL) { set_error("CQ row bit count exceeds the int32 interface"); return nullptr; }
    auto *m = new (std::nothrow) Matrix();
    if (!m) { set_error("out of host memory"); return nullptr; }
    m->sdot = sdot;
    CQDevice &w = m->w;
    w.out = out; w.in = in; w.bits = bits; w.group = group; w.padded = (int)padded;
    w.groups = (int)(padded / group); w.storage_bits = sbits; w.rowbytes = (int)(padded * sbits / 8);
    const int ncb = bits == 5 ? 3 : 1 << bits;
    for (int i = 0; i < 16; ++i) w.lut[i] = 0.f;
    if (bits == 5) {
        // crumb 0 -> cb[1], 1 -> cb[2], 3 -> cb[0] (needle2/csrc/cq.cpp:71-74)
        w.lut[0] = cb[1]; w.lut[1] = cb[2]; w.lut[3] = cb[0];
    } else {
        for (int i = 0; i < ncb; ++i) w.lut[i] = cb[i];
    }
    // SDOT weight side, as SdotCQ::SdotCQ (needle2/csrc/sdot.cpp:38-42).
    float maximum = 0.f;
    for (int i = 0; i < ncb; ++i) maximum = std::max(maximum, std::fabs(cb[i]));
    const float cs = maximum > 0 ? maximum / 127 : 1;
    int8_t cent[16] = {};
    if (bits == 2 || bits == 4)
        for (int i = 0; i < (1 << bits); ++i)
            cent[i] = (int8_t)std::min(127.f, std::max(-127.f, std::nearbyint(cb[i] / cs)));
    std::memcpy(w.ctab, cent, 16);
    w.centroid_scale = cs;
    // Sign split of the CQ4 int8 table (any sorted codebook with eight
    // non-positive and eight non-negative centroids): the decode then needs
    // two byte permutes per four elements, one per sign.
    w.split = 0;
    w.ntab[0] = w.ntab[1] = w.ptab[0] = w.ptab[1] = 0;
    if (bits == 4) {
        bool ok = true;
        uint8_t nb[8], pb[8];
        for (int i = 0; i < 8; ++i) {
            ok = ok && cent[i] <= 0 && cent[8 + i] >= 0;
            nb[i] = (uint8_t)(-cent[i]);
            pb[i] = (uint8_t)cent[8 + i];
        }
        if (ok) {
            w.split = 1;
            std::memcpy(w.ntab, nb, 8);
            std::memcpy(w.ptab, pb, 8);
        }
    }

    cudaGetDevice(&m->device);
    const size_t pbytes = (size_t)out * w.rowbytes, nbytes = sizeof(uint16_t) * (size_t)out * w.groups;
    cudaError_t e = cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaMalloc(&m->d_packed, pbytes + 64);
    if (e == cudaSuccess) e = cudaMalloc(&m->d_norms, nbytes + 64);
    if (e == cudaSuccess) e = cudaMemcpy(m->d_packed, packed, pbytes, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemset(m->d_packed + pbytes, 0, 64);
    if (e == cudaSuccess) e = cudaMemcpy(m->d_norms, norms, nbytes, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        set_error(std::string("CQ device upload failed: ") + cudaGetErrorString(e));
        delete m;
        return nullptr;
    }
    w.packed = m->d_packed;
    w.norms = m->d_norms;
    w.norms8 = m->d_norms;
    if (sdot && w.groups % 8) {
        // int8 kernels fetch the norms of eight groups at a time
        const int g8 = (w.groups + 7) / 8 * 8;
        std::vector<uint16_t> padded8((size_t)out * g8, 0);
        for (int r = 0; r < out; ++r)
            std::memcpy(&padded8[(size_t)r * g8], norms + (size_t)r * w.groups, sizeof(uint16_t) * w.groups);
        e = cudaMalloc(&m->d_norms8, sizeof(uint16_t) * padded8.size());
        if (e == cudaSuccess)
            e = cudaMemcpy(m->d_norms8, padded8.data(), sizeof(uint16_t) * padded8.size(), cudaMemcpyHostToDevice);
        if (e != cudaSuccess) {
            set_error(std::string("CQ device upload failed: ") + cudaGetErrorString(e));
            delete m;
            return nullptr;
        }
        w.norms8 = m->d_norms8;
    }
    if (sdot && (bits == 2 || bits == 4) && (group == 64 || group == 128 || group == 256)) {
        // fragment-order copy, repacked on the device from the row-major upload
        const size_t fb = nb200::frag_bytes(out, w.groups, group, bits), fnc = nb200::frag_norm_count(out, w.groups);
        e = cudaMalloc(&m->d_frag, fb);
        if (e == cudaSuccess) e = cudaMalloc(&m->d_normsF, sizeof(uint16_t) * fnc);
        bool ok = e == cudaSuccess && nb200::build_frag_layout(m->d_packed, m->d_norms, out, w.groups, group, bits,
                                                                w.rowbytes, m->d_frag, m->d_normsF, m->stream);
        if (ok) ok = cudaStreamSynchronize(m->stream) == cudaSuccess;
        if (!ok) {
            if (e != cudaSuccess) set_error(std::string("CQ device upload failed: ") + cudaGetErrorString(e));
            delete m;
            return nullptr;
        }
        w.frag = m->d_frag;
        w.normsF = m->d_normsF;
    }
    if (!sdot && (bits == 2 || bits == 4) && (group == 64 || group == 128 || group == 256) && w.rowbytes % 16 == 0) {
        // row-block copy for the FP32 decode GEMV, repacked on the device
        e = cudaMalloc(&m->d_blocked, nb200::blocked_bytes(out, w.groups, group, bits));
        if (e == cudaSuccess) e = cudaMalloc(&m->d_normsB, sizeof(uint16_t) * nb200::blocked_norm_count(out, w.groups));
        bool ok = e == cudaSuccess && nb200::build_blocked_layout(m->d_packed, m->d_norms, out, w.groups, group, bits,
                                                                   w.rowbytes, m->d_blocked, m->d_normsB, m->stream);
        if (ok) ok = cudaStreamSynchronize(m->stream) == cudaSuccess;
        if (!ok) {
            if (e != cudaSuccess) set_error(std::string("CQ device upload failed: ") + cudaGetErrorString(e));
            delete m;
            return nullptr;
        }
        w.blocked = m->d_blocked;
        w.normsB = m->d_normsB;
    }
    return m;
}

// Enqueue y = W x on `st` for device x[batch][in] -> y[batch][out].
// int8 products of a prepared batch: the tensor-core GEMM from kGemmMinRows
// activation rows on (decoding the matrix for it at the first such call), the
// GEMV otherwise and whenever the int32 group dots are exported.
// Decoded int8 weights and group scales for the prefill GEMM, made at the first use.
bool ensure_gemm_copy(Matrix *m, cudaStream_t st) {
    const CQDevice &w = m->w;
    if (!m->d_w8) {
        cudaError_t e = cudaMalloc(&m->d_w8, gemm_w8_bytes(w.out, w.padded));
        if (e == cudaSuccess) e = cudaMalloc(&m->d_nsT, sizeof(float) * gemm_ns_count(w.out, w.groups));
        if (e != cudaSuccess) {
            if (m->d_w8) cudaFree(m->d_w8);
            if (m->d_nsT) cudaFree(m->d_nsT);
            m->d_w8 = nullptr;
            m->d_nsT = nullptr;
            set_error(std::string("prefill weight allocation failed: ") + cudaGetErrorString(e));
            return false;
        }
        if (!gemm_prepare(w.packed, w.norms, w.out, w.groups, w.group, w.bits, w.rowbytes, w.padded, w.ctab,
                          w.centroid_scale, m->d_w8, m->d_nsT, st)) {
            // leave no half-made copy behind: the next call prepares again
            cudaFree(m->d_w8);
            cudaFree(m->d_nsT);
            m->d_w8 = nullptr;
            m->d_nsT = nullptr;
            return false;
        }
    }
    return true;
}

bool sdot_multiply(Matrix *m, const int8_t *q, const float *xs, int batch, float *y, int32_t *partials,
                   cudaStream_t st) {
    const CQDevice &w = m->w;
    if (partials || batch < kGemmMinRows || !gemm_supported(w.bits, w.group, w.padded))
        return launch_gemv_i8(w, q, xs, batch, y, w.out, partials, st);
    if (!ensure_gemm_copy(m, st)) return false;
    return launch_gemm_i8(q, xs, batch, m->d_w8, m->d_nsT, w.out, w.padded, w.groups, y, w.out, st);
}

// y[batch][out] written into each of dsts[0..ndst) with row stride ldy (for
// instance this matrix's column range of every rank's [batch][N] output): the
// GEMM writes all destinations from its epilogue; smaller batches run the GEMV
// into scratch and copy it to each destination.
bool sdot_multiply_to(Matrix *m, const int8_t *q, const float *xs, int batch, float *const *dsts, int ndst, int ldy,
                      cudaStream_t st) {
    const CQDevice &w = m->w;
    if (batch >= kGemmMinRows && gemm_supported(w.bits, w.group, w.padded)) {
        if (!ensure_gemm_copy(m, st)) return false;
        return launch_gemm_i8_multi(q, xs, batch, m->d_w8, m->d_nsT, w.out, w.padded, w.groups, dsts, ndst, ldy, st);
    }
    if (!m->y.reserve((size_t)batch * w.out)) return false;
    if (!launch_gemv_i8(w, q, xs, batch, m->y.ptr, w.out, nullptr, st)) return false;
    for (int i = 0; i < ndst; ++i)
        NB_CUDA_TRY(cudaMemcpy2DAsync(dsts[i], sizeof(float) * ldy, m->y.ptr, sizeof(float) * w.out,
                                      sizeof(float) * w.out, batch, cudaMemcpyDeviceToDevice, st));
    return true;
}

// FP32 mode, y[batch][out] from rotated activations: the tensor-core GEMM from
// kGemmMinRows rows on (bf16 hi/lo weights made at the first such call; the
// activations split here unless a_hilo already holds them), the GEMV otherwise.
// FP32 mode: bf16 hi/lo weights for the prefill GEMM, made at the first use.
bool ensure_f32_copy(Matrix *m, cudaStream_t st) {
    const CQDevice &w = m->w;
    if (m->d_whl) return true;
    const cudaError_t e = cudaMalloc(&m->d_whl, sizeof(uint16_t) * gemm_f32_weight_elems(w.out, w.padded));
    if (e != cudaSuccess) {
        m->d_whl = nullptr;
        set_error(std::string("prefill weight allocation failed: ") + cudaGetErrorString(e));
        return false;
    }
    if (!gemm_f32_prepare(w.packed, w.norms, w.out, w.groups, w.group, w.storage_bits, w.rowbytes, w.padded, w.lut,
                          m->d_whl, st)) {
        cudaFree(m->d_whl);
        m->d_whl = nullptr;
        return false;
    }
    return true;
}

bool f32_multiply(Matrix *m, const float *rot, int batch, float *y, cudaStream_t st,
                  const uint16_t *a_hilo = nullptr) {
    const CQDevice &w = m->w;
    if (batch < kGemmMinRows || !gemm_f32_supported(w.storage_bits, w.padded))
        return launch_gemv_f32(w, rot, batch, y, w.out, st);
    if (!ensure_f32_copy(m, st)) return false;
    if (!a_hilo) {
        if (!m->ahl.reserve(2 * (size_t)batch * w.padded)) return false;
        if (!launch_split_bf16(rot, (long long)batch * w.padded, m->ahl.ptr, st)) return false;
        a_hilo = m->ahl.ptr;
    }
    return launch_gemm_f32x3(a_hilo, batch, m->d_whl, w.out, w.padded, y, w.out, st);
}

bool run_linear_device(Matrix *m, const float *x, float *y, int batch, cudaStream_t st, int32_t *partials) {
    m->prepared = 0;
    if (batch <= 0) return true;
    const CQDevice &w = m->w;
    if (!m->sdot && batch >= kGemmMinRows && gemm_f32_supported(w.storage_bits, w.padded) && w.group <= 1024) {
        // prefill-sized FP32 batch: the rotation writes the GEMM's bf16 operands directly
        if (!m->ahl.reserve(2 * (size_t)batch * w.padded)) return false;
        if (!launch_rotate_hilo(w, x, batch, m->ahl.ptr, st)) return false;
        return f32_multiply(m, nullptr, batch, y, st, m->ahl.ptr);
    }
    if (!m->sdot) {
        if (!m->rot.reserve((size_t)batch * w.padded)) return false;
        if (!launch_rotate(w, x, batch, m->rot.ptr, st)) return false;
        return f32_multiply(m, m->rot.ptr, batch, y, st);
    }
    if (!m->q.reserve((size_t)batch * w.padded) || !m->xs.reserve((size_t)batch * w.groups)) return false;
    if (!launch_quantize(w, x, batch, m->q.ptr, m->xs.ptr, st)) return false;
    return sdot_multiply(m, m->q.ptr, m->xs.ptr, batch, y, partials, st);
}

bool run_linear_host(Matrix *m, const float *x, float *y, int batch, int32_t *partials_host, int8_t *q_host,
                     float *scales_host) {
    clear_error();
    if (!m) { set_error("null handle"); return false; }
    if (batch < 0) { set_error("negative batch"); return false; }
    if (batch == 0) return true;
    if ((long long)batch * m->w.out > 0x7fffffffLL) { set_error("batch output count exceeds the int32 interface"); return false; }
    NB_CUDA_TRY(cudaSetDevice(m->device));
    const CQDevice &w = m->w;
    const cudaStream_t st = m->stream;
    if (!m->x.reserve((size_t)batch * w.in) || !m->y.reserve((size_t)batch * w.out)) return false;
    int32_t *dpart = nullptr;
    if (partials_host) {
        if (!m->partials.reserve((size_t)batch * w.out * w.groups)) return false;
        dpart = m->partials.ptr;
    }
    NB_CUDA_TRY(cudaMemcpyAsync(m->x.ptr, x, sizeof(float) * (size_t)batch * w.in, cudaMemcpyHostToDevice, st));
    if (!run_linear_device(m, m->x.ptr, m->y.ptr, batch, st, dpart)) return false;
    if (y) NB_CUDA_TRY(cudaMemcpyAsync(y, m->y.ptr, sizeof(float) * (size_t)batch * w.out, cudaMemcpyDeviceToHost, st));
    if (partials_host)
        NB_CUDA_TRY(cudaMemcpyAsync(partials_host, dpart, sizeof(int32_t) * (size_t)batch * w.out * w.groups,
                                    cudaMemcpyDeviceToHost, st));
    std::vector<int8_t> qtmp;
    if (q_host) {
        qtmp.resize((size_t)batch * w.padded);
        NB_CUDA_TRY(cudaMemcpyAsync(qtmp.data(), m->q.ptr, qtmp.size(), cudaMemcpyDeviceToHost, st));
    }
    if (scales_host)
        NB_CUDA_TRY(cudaMemcpyAsync(scales_host, m->xs.ptr, sizeof(float) * (size_t)batch * w.groups,
                                    cudaMemcpyDeviceToHost, st));
    NB_CUDA_TRY(cudaStreamSynchronize(st));
    if (q_host) {
        // undo the CQ2 bit-plane order so callers see natural element order
        for (size_t i = 0; i < qtmp.size(); ++i) {
            size_t e = i % w.padded, base = i - e;
            size_t d = w.bits == 2 ? ((e & ~size_t(15)) | ((e & 1) ? 8 + ((e & 15) >> 1) : ((e & 15) >> 1))) : e;
            q_host[base + e] = qtmp[base + d];
        }
    }
    return true;
}

}  // namespace
}  // namespace nb200

namespace nb200 {

const CQDevice *handle_matrix(void *handle) { return handle ? &static_cast<Matrix *>(handle)->w : nullptr; }
bool handle_is_sdot(void *handle) { return handle && static_cast<Matrix *>(handle)->sdot; }
int handle_device(void *handle) { return static_cast<Matrix *>(handle)->device; }

bool handle_prepare(void *handle, const float *x, int batch, const float **rot, const int8_t **q, const float **xs,
                    cudaStream_t st) {
    auto *m = static_cast<Matrix *>(handle);
    const CQDevice &w = m->w;
    m->prepared = 0;
    if (m->sdot) {
        if (!m->q.reserve((size_t)batch * w.padded) || !m->xs.reserve((size_t)batch * w.groups)) return false;
        if (!launch_quantize(w, x, batch, m->q.ptr, m->xs.ptr, st)) return false;
        if (q) *q = m->q.ptr;
        if (xs) *xs = m->xs.ptr;
    } else {
        if (!m->rot.reserve((size_t)batch * w.padded)) return false;
        if (!launch_rotate(w, x, batch, m->rot.ptr, st)) return false;
        if (rot) *rot = m->rot.ptr;
    }
    m->prepared = batch;
    return true;
}

void *handle_make_sdot(void *cq) {
    auto *m = static_cast<Matrix *>(cq);
    const CQDevice &w = m->w;
    if (m->sdot) { set_error("handle is already an int8 matrix"); return nullptr; }
    if (cudaSetDevice(m->device) != cudaSuccess) { set_error("cudaSetDevice failed"); return nullptr; }
    std::vector<uint8_t> packed((size_t)w.out * w.rowbytes);
    std::vector<uint16_t> norms((size_t)w.out * w.groups);
    if (cudaStreamSynchronize(m->stream) != cudaSuccess ||
        cudaMemcpy(packed.data(), w.packed, packed.size(), cudaMemcpyDeviceToHost) != cudaSuccess ||
        cudaMemcpy(norms.data(), w.norms, 2 * norms.size(), cudaMemcpyDeviceToHost) != cudaSuccess) {
        set_error("reading back the CQ matrix failed");
        return nullptr;
    }
    float cb[16] = {};
    const int ncb = w.bits == 5 ? 3 : 1 << w.bits;
    for (int i = 0; i < ncb; ++i) cb[i] = w.lut[i];
    return create_matrix(packed.data(), norms.data(), w.out, w.in, w.bits, w.group, cb, true);
}

}  // namespace nb200

using nb200::Matrix;

extern "C" {

const char *needle2_native_features() { return "cuda-sm100a;float32-accumulate;direct-packed-cq;sdot-int8"; }

const char *needle2_b200_error() { return nb200::last_error(); }

void *needle2_cq_create(const uint8_t *p, const uint16_t *n, int out, int in, int bits, int group, const float *cb) {
    return nb200::create_matrix(p, n, out, in, bits, group, cb, false);
}

void needle2_cq_destroy(void *handle) { delete static_cast<Matrix *>(handle); }

int needle2_cq_linear_checked(void *handle, const float *x, float *y, int batch) {
    auto *m = static_cast<Matrix *>(handle);
    if (m && m->sdot) { nb200::set_error("handle is an SDOT matrix"); return -1; }
    return nb200::run_linear_host(m, x, y, batch, nullptr, nullptr, nullptr) ? 0 : -1;
}

void needle2_cq_linear(void *handle, const float *x, float *y, int batch, int threads) {
    (void)threads;
    needle2_cq_linear_checked(handle, x, y, batch);
}

void needle2_cq_linear_lookup(void *handle, const float *x, float *y, int batch, int threads, int mode) {
    (void)mode;
    needle2_cq_linear(handle, x, y, batch, threads);
}

namespace nb200 {
namespace {

// Matrices that can share one prepared activation and one fused launch.
bool fusable(Matrix *const *ms, int count) {
    if (count < 1) return false;
    const CQDevice &a = ms[0]->w;
    if (!gemv_max_rows(a.bits, a.group, a.groups, ms[0]->sdot)) return false;
    for (int i = 0; i < count; ++i) {
        if (!ms[i]) return false;
        const CQDevice &w = ms[i]->w;
        if (ms[i]->sdot != ms[0]->sdot || ms[i]->device != ms[0]->device || w.in != a.in ||
            w.group != a.group || w.bits != a.bits || std::memcmp(w.lut, a.lut, sizeof(a.lut)) ||
            std::memcmp(w.ctab, a.ctab, sizeof(a.ctab)) || w.centroid_scale != a.centroid_scale)
            return false;
    }
    return true;
}

bool multiply_many(Matrix *const *ms, int count, float *const *ys, int batch, cudaStream_t st);

// y_i[batch][out_i] = W_i x for device x / y_i: one prepare (on the first
// matrix's scratch), then fused launches of up to kGemvMaxMats matrices.
bool many_device(Matrix *const *ms, int count, const float *x, float *const *ys, int batch, cudaStream_t st) {
    if (batch <= 0 || count <= 0) return true;
    if (!fusable(ms, count)) {
        for (int i = 0; i < count; ++i)
            if (!run_linear_device(ms[i], x, ys[i], batch, st, nullptr)) return false;
        return true;
    }
    Matrix *m0 = ms[0];
    const CQDevice &w = m0->w;
    const bool i8 = m0->sdot;
    if (!i8 && batch >= kGemmMinRows && gemm_f32_supported(w.storage_bits, w.padded) && w.group <= 1024) {
        // prefill-sized FP32 batch: rotate straight into the bf16 operands, one GEMM launch for every matrix
        if (!m0->ahl.reserve(2 * (size_t)batch * w.padded)) return false;
        if (!launch_rotate_hilo(w, x, batch, m0->ahl.ptr, st)) return false;
        m0->prepared = 0;   // the FP32 activations themselves were not kept
        std::vector<F32Out> outs(count);
        for (int i = 0; i < count; ++i) {
            if (!ensure_f32_copy(ms[i], st)) return false;
            outs[i] = F32Out{ms[i]->d_whl, ms[i]->w.out, ys[i], ms[i]->w.out};
        }
        return launch_gemm_f32x3_multi(m0->ahl.ptr, batch, w.padded, outs.data(), count, st);
    }
    if (i8) {
        if (!m0->q.reserve((size_t)batch * w.padded) || !m0->xs.reserve((size_t)batch * w.groups)) return false;
        if (!launch_quantize(w, x, batch, m0->q.ptr, m0->xs.ptr, st)) return false;
    } else {
        if (!m0->rot.reserve((size_t)batch * w.padded)) return false;
        if (!launch_rotate(w, x, batch, m0->rot.ptr, st)) return false;
    }
    m0->prepared = batch;
    return multiply_many(ms, count, ys, batch, st);
}

// Fused launches from the activations prepared on ms[0].
bool multiply_many(Matrix *const *ms, int count, float *const *ys, int batch, cudaStream_t st) {
    Matrix *m0 = ms[0];
    const CQDevice &w = m0->w;
    const bool i8 = m0->sdot;
    if (batch > m0->prepared) { set_error("multiply batch exceeds the prepared batch"); return false; }
    if (i8 && batch >= kGemmMinRows && gemm_supported(w.bits, w.group, w.padded)) {
        // prefill-sized batches: one tensor-core GEMM per matrix on the shared input
        for (int i = 0; i < count; ++i)
            if (!sdot_multiply(ms[i], m0->q.ptr, m0->xs.ptr, batch, ys[i], nullptr, st)) return false;
        return true;
    }
    if (!i8 && batch >= kGemmMinRows && gemm_f32_supported(w.storage_bits, w.padded)) {
        // FP32 prefill-sized batches: the activations split once, every matrix in one GEMM launch
        if (!m0->ahl.reserve(2 * (size_t)batch * w.padded)) return false;
        if (!launch_split_bf16(m0->rot.ptr, (long long)batch * w.padded, m0->ahl.ptr, st)) return false;
        std::vector<F32Out> outs(count);
        for (int i = 0; i < count; ++i) {
            if (!ensure_f32_copy(ms[i], st)) return false;
            outs[i] = F32Out{ms[i]->d_whl, ms[i]->w.out, ys[i], ms[i]->w.out};
        }
        return launch_gemm_f32x3_multi(m0->ahl.ptr, batch, w.padded, outs.data(), count, st);
    }
    const int cap = gemv_max_rows(w.bits, w.group, w.groups, i8);
    for (int i0 = 0; i0 < count; i0 += kGemvMaxMats) {
        const int n = std::min(kGemvMaxMats, count - i0);
        for (int r0 = 0; r0 < batch; r0 += cap) {
            GemvBatch b = single_batch(w);
            b.nmat = n;
            b.M = std::min(cap, batch - r0);
            for (int j = 0; j < n; ++j) {
                const CQDevice &wj = ms[i0 + j]->w;
                b.mat[j].packed = wj.packed;
                b.mat[j].norms = wj.norms;
                b.mat[j].norms8 = wj.norms8;
                b.mat[j].frag = wj.frag;
                b.mat[j].normsF = wj.normsF;
                b.mat[j].blocked = wj.blocked;
                b.mat[j].normsB = wj.normsB;
                b.mat[j].out = wj.out;
                b.mat[j].y = ys[i0 + j] + (size_t)r0 * wj.out;
            }
            if (i8) {
                b.q = m0->q.ptr + (size_t)r0 * w.padded;
                b.xs = m0->xs.ptr + (size_t)r0 * w.groups;
            } else {
                b.rot = m0->rot.ptr + (size_t)r0 * w.padded;
            }
            if (!launch_gemv(b, i8, st)) return false;
        }
    }
    return true;
}

// Host form: x[batch][in] -> ys[i][batch][out_i], synchronised.
bool many_host(Matrix *const *ms, int count, const float *x, float *const *ys, int batch) {
    clear_error();
    if (count <= 0 || batch <= 0) return true;
    for (int i = 0; i < count; ++i)
        if (!ms[i]) { set_error("null handle"); return false; }
    Matrix *m0 = ms[0];
    NB_CUDA_TRY(cudaSetDevice(m0->device));
    const cudaStream_t st = m0->stream;
    size_t total = 0;
    for (int i = 0; i < count; ++i) total += (size_t)batch * ms[i]->w.out;
    if (!m0->x.reserve((size_t)batch * m0->w.in) || !m0->y.reserve(total)) return false;
    const size_t xn = (size_t)batch * m0->w.in;
    if (is_pinned(x)) {
        NB_CUDA_TRY(cudaMemcpyAsync(m0->x.ptr, x, sizeof(float) * xn, cudaMemcpyHostToDevice, st));
    } else {
        if (!m0->hin.reserve(xn)) return false;
        NB_CUDA_TRY(cudaStreamSynchronize(st));   // the staging buffer may still feed an earlier copy
        std::memcpy(m0->hin.ptr, x, sizeof(float) * xn);
        NB_CUDA_TRY(cudaMemcpyAsync(m0->x.ptr, m0->hin.ptr, sizeof(float) * xn, cudaMemcpyHostToDevice, st));
    }
    // page-locked outputs: the kernels store the results straight into them
    std::vector<float *> dys(count);
    bool mapped = true;
    for (int i = 0; i < count && mapped; ++i) mapped = (dys[i] = mapped_host(ys[i])) != nullptr;
    if (mapped) {
        if (!many_device(ms, count, m0->x.ptr, dys.data(), batch, st)) return false;
        NB_CUDA_TRY(cudaStreamSynchronize(st));
        return true;
    }
    size_t off = 0;
    for (int i = 0; i < count; ++i) {
        dys[i] = m0->y.ptr + off;
        off += (size_t)batch * ms[i]->w.out;
    }
    if (!many_device(ms, count, m0->x.ptr, dys.data(), batch, st)) return false;
    // pageable outputs: one transfer of all of them into pinned staging, then host copies
    if (!m0->hout.reserve(total)) return false;
    NB_CUDA_TRY(cudaMemcpyAsync(m0->hout.ptr, m0->y.ptr, sizeof(float) * total, cudaMemcpyDeviceToHost, st));
    NB_CUDA_TRY(cudaStreamSynchronize(st));
    off = 0;
    for (int i = 0; i < count; ++i) {
        const size_t n = (size_t)batch * ms[i]->w.out;
        std::memcpy(ys[i], m0->hout.ptr + off, sizeof(float) * n);
        off += n;
    }
    return true;
}

}  // namespace

// (this block sits inside the file's extern "C" region; these are C++ functions)
extern "C++" {
bool handle_hilo_gemm(void *const *hs, int count, int batch, int *group, float *scale) {
    if (count < 1 || batch < kGemmMinRows) return false;
    std::vector<Matrix *> ms(count);
    for (int i = 0; i < count; ++i) ms[i] = static_cast<Matrix *>(hs[i]);
    if (!ms[0] || ms[0]->sdot || !fusable(ms.data(), count)) return false;
    const CQDevice &w = ms[0]->w;
    if (!gemm_f32_supported(w.storage_bits, w.padded) || w.group > 1024 || w.padded != w.in) return false;
    if (group) *group = w.group;
    if (scale) *scale = 1.0f / sqrtf((float)w.group);   // the rotation's scale (launch_rotate_impl)
    return true;
}

bool handle_many_hilo(void *const *hs, int count, const uint16_t *a_hilo, float *const *ys, int batch,
                      cudaStream_t st, const QkvgEpilogue *epi, bool *epi_done, const KParts *kp) {
    if (epi_done) *epi_done = false;
    if (kp && kp->parts) *kp->parts = 1;
    if (!handle_hilo_gemm(hs, count, batch, nullptr, nullptr)) {
        set_error("these matrices do not take pre-split bf16 activations");
        return false;
    }
    std::vector<F32Out> outs(count);
    for (int i = 0; i < count; ++i) {
        auto *m = static_cast<Matrix *>(hs[i]);
        m->prepared = 0;
        if (!ensure_f32_copy(m, st)) return false;
        outs[i] = F32Out{m->d_whl, m->w.out, ys[i], m->w.out};
    }
    return launch_gemm_f32x3_multi(a_hilo, batch, static_cast<Matrix *>(hs[0])->w.padded, outs.data(), count, st,
                                   epi, epi_done, kp);
}
}  // extern "C++"

}  // namespace nb200

void needle2_cq_linear_many(void *const *handles, int count, const float *x, float *const *ys, int threads,
                            int mode) {
    (void)mode;
    (void)threads;
    std::vector<Matrix *> ms(count > 0 ? count : 0);
    for (int i = 0; i < count; ++i) {
        ms[i] = static_cast<Matrix *>(handles[i]);
        if (ms[i] && ms[i]->sdot) { nb200::set_error("needle2_cq_linear_many takes FP32-mode handles"); return; }
    }
    nb200::many_host(ms.data(), count, x, ys, 1);
}

int needle2_cq_linear_many_checked(void *const *handles, int count, const float *x, float *const *ys, int batch,
                                   int sdot) {
    std::vector<Matrix *> ms(count > 0 ? count : 0);
    for (int i = 0; i < count; ++i) {
        ms[i] = static_cast<Matrix *>(handles[i]);
        if (!ms[i] || ms[i]->sdot != (sdot != 0)) { nb200::set_error("null or wrong-kind handle"); return -1; }
    }
    return nb200::many_host(ms.data(), count, x, ys, batch) ? 0 : -1;
}

int needle2_cq_multiply_many_device(void *const *handles, int count, float *const *ys, int batch, int sdot,
                                    void *stream) {
    nb200::clear_error();
    std::vector<Matrix *> ms(count > 0 ? count : 0);
    for (int i = 0; i < count; ++i) {
        ms[i] = static_cast<Matrix *>(handles[i]);
        if (!ms[i] || ms[i]->sdot != (sdot != 0)) { nb200::set_error("null or wrong-kind handle"); return -1; }
    }
    if (count <= 0 || batch <= 0) return 0;
    if (!nb200::fusable(ms.data(), count)) { nb200::set_error("matrices cannot share one launch"); return -1; }
    if (cudaSetDevice(ms[0]->device) != cudaSuccess) { nb200::set_error("cudaSetDevice failed"); return -1; }
    return nb200::multiply_many(ms.data(), count, ys, batch, static_cast<cudaStream_t>(stream)) ? 0 : -1;
}

int needle2_cq_linear_many_device(void *const *handles, int count, const float *x, float *const *ys, int batch,
                                  int sdot, void *stream) {
    nb200::clear_error();
    std::vector<Matrix *> ms(count > 0 ? count : 0);
    for (int i = 0; i < count; ++i) {
        ms[i] = static_cast<Matrix *>(handles[i]);
        if (!ms[i] || ms[i]->sdot != (sdot != 0)) { nb200::set_error("null or wrong-kind handle"); return -1; }
    }
    if (count > 0 && cudaSetDevice(ms[0]->device) != cudaSuccess) { nb200::set_error("cudaSetDevice failed"); return -1; }
    return nb200::many_device(ms.data(), count, x, ys, batch, static_cast<cudaStream_t>(stream)) ? 0 : -1;
}

void needle2_cq_rows(void *handle, const int64_t *ids, float *y, int count) {
    nb200::clear_error();
    auto *m = static_cast<Matrix *>(handle);
    if (!m || count <= 0) return;
    for (int i = 0; i < count; ++i)
        if (ids[i] < 0 || ids[i] >= m->w.out) { nb200::set_error("CQ row index outside matrix"); return; }
    if (cudaSetDevice(m->device) != cudaSuccess) { nb200::set_error("cudaSetDevice failed"); return; }
    if (!m->ids.reserve((size_t)count) || !m->y.reserve((size_t)count * m->w.in)) return;
    cudaStream_t st = m->stream;
    cudaError_t e = cudaMemcpyAsync(m->ids.ptr, ids, sizeof(int64_t) * count, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess && !nb200::launch_rows(m->w, m->ids.ptr, count, m->y.ptr, st)) return;
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(y, m->y.ptr, sizeof(float) * (size_t)count * m->w.in, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) nb200::set_error(std::string("needle2_cq_rows: ") + cudaGetErrorString(e));
}

int needle2_sdot_supported() { return 1; }

void *needle2_sdot_create(const uint8_t *p, const uint16_t *n, int out, int in, int bits, int group, const float *cb) {
    return nb200::create_matrix(p, n, out, in, bits, group, cb, true);
}

void needle2_sdot_destroy(void *handle) { delete static_cast<Matrix *>(handle); }

int needle2_sdot_linear_checked(void *handle, const float *x, float *y, int batch) {
    auto *m = static_cast<Matrix *>(handle);
    if (m && !m->sdot) { nb200::set_error("handle is not an SDOT matrix"); return -1; }
    return nb200::run_linear_host(m, x, y, batch, nullptr, nullptr, nullptr) ? 0 : -1;
}

void needle2_sdot_linear(void *handle, const float *x, float *y, int batch, int threads) {
    (void)threads;
    needle2_sdot_linear_checked(handle, x, y, batch);
}

int needle2_sdot_debug(void *handle, const float *x, int batch, float *y, int32_t *partials, int8_t *q,
                       float *scales) {
    auto *m = static_cast<Matrix *>(handle);
    if (!m || !m->sdot) { nb200::set_error("handle is not an SDOT matrix"); return -1; }
    return nb200::run_linear_host(m, x, y, batch, partials, q, scales) ? 0 : -1;
}

static int linear_device(void *handle, const float *x, float *y, int batch, void *stream, bool sdot) {
    nb200::clear_error();
    auto *m = static_cast<Matrix *>(handle);
    if (!m) { nb200::set_error("null handle"); return -1; }
    if (m->sdot != sdot) { nb200::set_error(sdot ? "handle is not an SDOT matrix" : "handle is an SDOT matrix"); return -1; }
    if (batch < 0) { nb200::set_error("negative batch"); return -1; }
    if (cudaSetDevice(m->device) != cudaSuccess) { nb200::set_error("cudaSetDevice failed"); return -1; }
    return nb200::run_linear_device(m, x, y, batch, static_cast<cudaStream_t>(stream), nullptr) ? 0 : -1;
}

int needle2_cq_linear_device(void *handle, const float *x, float *y, int batch, void *stream) {
    return linear_device(handle, x, y, batch, stream, false);
}

int needle2_sdot_linear_device(void *handle, const float *x, float *y, int batch, void *stream) {
    return linear_device(handle, x, y, batch, stream, true);
}

// Two-phase form of the device entry points: prepare (rotate, or rotate and
// quantise) the activations into the handle's scratch, then multiply.  The
// split follows SdotCQ::prepare / SdotCQ::multiply (needle2/csrc/sdot.cpp:47,338).
static int prepare_device(void *handle, const float *x, int batch, void *stream, bool sdot) {
    nb200::clear_error();
    auto *m = static_cast<Matrix *>(handle);
    if (!m || m->sdot != sdot) { nb200::set_error("null or wrong-kind handle"); return -1; }
    if (batch < 0) { nb200::set_error("negative batch"); return -1; }
    if (cudaSetDevice(m->device) != cudaSuccess) { nb200::set_error("cudaSetDevice failed"); return -1; }
    const nb200::CQDevice &w = m->w;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    m->prepared = 0;
    if (batch == 0) return 0;
    if (sdot) {
        if (!m->q.reserve((size_t)batch * w.padded) || !m->xs.reserve((size_t)batch * w.groups)) return -1;
        if (!nb200::launch_quantize(w, x, batch, m->q.ptr, m->xs.ptr, st)) return -1;
    } else {
        if (!m->rot.reserve((size_t)batch * w.padded)) return -1;
        if (!nb200::launch_rotate(w, x, batch, m->rot.ptr, st)) return -1;
    }
    m->prepared = batch;
    return 0;
}

static int multiply_device(void *handle, float *y, int batch, void *stream, bool sdot) {
    nb200::clear_error();
    auto *m = static_cast<Matrix *>(handle);
    if (!m || m->sdot != sdot) { nb200::set_error("null or wrong-kind handle"); return -1; }
    if (batch < 0 || batch > m->prepared) { nb200::set_error("multiply batch exceeds the prepared batch"); return -1; }
    if (cudaSetDevice(m->device) != cudaSuccess) { nb200::set_error("cudaSetDevice failed"); return -1; }
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const nb200::CQDevice &w = m->w;
    bool ok = sdot ? nb200::sdot_multiply(m, m->q.ptr, m->xs.ptr, batch, y, nullptr, st)
                   : nb200::f32_multiply(m, m->rot.ptr, batch, y, st);
    return ok ? 0 : -1;
}

int needle2_cq_prepare_device(void *h, const float *x, int batch, void *stream) {
    return prepare_device(h, x, batch, stream, false);
}
int needle2_cq_multiply_device(void *h, float *y, int batch, void *stream) {
    return multiply_device(h, y, batch, stream, false);
}
int needle2_sdot_prepare_device(void *h, const float *x, int batch, void *stream) {
    return prepare_device(h, x, batch, stream, true);
}
int needle2_sdot_multiply_device(void *h, float *y, int batch, void *stream) {
    return multiply_device(h, y, batch, stream, true);
}

int needle2_sdot_multiply_gather_device(void *h, float *const *dsts, int ndst, int ldy, int batch, void *stream) {
    nb200::clear_error();
    auto *m = static_cast<Matrix *>(h);
    if (!m || !m->sdot) { nb200::set_error("null or wrong-kind handle"); return -1; }
    if (!dsts || ndst < 1 || ndst > nb200::kMaxGemmOutputs) { nb200::set_error("1 to 8 output buffers"); return -1; }
    if (ldy < m->w.out) { nb200::set_error("ldy is smaller than the matrix's out"); return -1; }
    if (batch < 0 || batch > m->prepared) { nb200::set_error("multiply batch exceeds the prepared batch"); return -1; }
    for (int i = 0; i < ndst; ++i)
        if (!dsts[i]) { nb200::set_error("null output buffer"); return -1; }
    if (batch == 0) return 0;
    if (cudaSetDevice(m->device) != cudaSuccess) { nb200::set_error("cudaSetDevice failed"); return -1; }
    return nb200::sdot_multiply_to(m, m->q.ptr, m->xs.ptr, batch, dsts, ndst, ldy, static_cast<cudaStream_t>(stream))
               ? 0
               : -1;
}

int needle2_b200_argmax_device(const float *logits, int rows, int vocab, int ld, int *out, void *stream) {
    nb200::clear_error();
    if (rows < 0 || vocab <= 0 || ld < vocab || (rows && (!logits || !out))) {
        nb200::set_error("argmax: bad arguments");
        return -1;
    }
    return nb200::launch_argmax(logits, rows, vocab, ld, out, static_cast<cudaStream_t>(stream)) ? 0 : -1;
}

int needle2_b200_activation_quant_device(float *x, int rows, int dim, int bits, void *stream) {
    nb200::clear_error();
    if (rows < 0 || dim < 0 || bits < 0 || bits > 16 || (rows && dim && !x)) {
        nb200::set_error("activation_quant: bad arguments");
        return -1;
    }
    return nb200::launch_activation_quant(x, rows, dim, bits, static_cast<cudaStream_t>(stream)) ? 0 : -1;
}

int needle2_b200_activation_quant(float *x, int rows, int dim, int bits) {
    nb200::clear_error();
    if (rows < 0 || dim < 0 || bits < 0 || bits > 16 || (rows && dim && !x)) {
        nb200::set_error("activation_quant: bad arguments");
        return -1;
    }
    if (!rows || !dim || !bits) return 0;
    const size_t bytes = sizeof(float) * (size_t)rows * dim;
    float *d = nullptr;
    if (cudaMalloc(&d, bytes) != cudaSuccess) { nb200::set_error("cudaMalloc failed"); return -1; }
    bool ok = cudaMemcpy(d, x, bytes, cudaMemcpyHostToDevice) == cudaSuccess;
    if (!ok) nb200::set_error("activation_quant: host-to-device copy failed");
    ok = ok && nb200::launch_activation_quant(d, rows, dim, bits, nullptr);
    if (ok && cudaMemcpy(x, d, bytes, cudaMemcpyDeviceToHost) != cudaSuccess) {
        nb200::set_error("activation_quant: device-to-host copy failed");
        ok = false;
    }
    cudaFree(d);
    return ok ? 0 : -1;
}

int needle2_b200_device_fault() { return nb200::read_and_clear_gemv_fault(); }

int needle2_cq_geometry(void *handle, int *g) {
    auto *m = static_cast<Matrix *>(handle);
    if (!m || !g) { nb200::set_error("null handle"); return -1; }
    g[0] = m->w.out; g[1] = m->w.in; g[2] = m->w.bits; g[3] = m->w.group; g[4] = m->w.padded; g[5] = m->w.groups;
    return 0;
}

}  // extern "C"

// ---- SDOT on device pointers without any device allocation -----------------
//
// needle2_sdot_linear_device keeps the quantised activations in scratch that
// the handle allocates (cudaMalloc) on first use and grows with the batch.
// Callers that may not allocate device memory while they run -- a serving
// loop on a memory pool sized up front, code that must not trigger the
// device-wide synchronisation cudaMalloc/cudaFree imply -- use
// needle2_sdot_linear_device_noalloc instead: its scratch is the two
// fixed-size arrays below, which exist once on every device that loads this
// library.  Neither array needs initial contents: each call's quantiser
// writes every activation byte and scale that the same call's GEMV reads.

namespace nb200 {

constexpr size_t kNoAllocActivationBytes = size_t(1) << 20;   // batch * padded int8 activations
constexpr size_t kNoAllocScales = size_t(1) << 14;            // batch * groups float scales

static __device__ __align__(256) int8_t g_noalloc_q[kNoAllocActivationBytes];
static __device__ __align__(256) float g_noalloc_xs[kNoAllocScales];

namespace {

struct NoAllocScratch {
    int8_t *q = nullptr;
    float *xs = nullptr;
};

// Unique id of the calling thread's current CUDA context (cuCtxGetId, reached
// through the runtime's driver entry points so the library links no libcuda),
// or 0 when it cannot be read.  A device reset destroys the primary context
// and the next call creates a new one with a new id, in which the library's
// module -- and with it the scratch arrays -- is loaded again, possibly at
// other addresses.
unsigned long long current_context_id() {
    using GetCurrent = int (*)(void **);
    using GetId = int (*)(void *, unsigned long long *);
    static GetCurrent get_current = nullptr;
    static GetId get_id = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        cudaDriverEntryPointQueryResult q;
        void *fn = nullptr;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_current = reinterpret_cast<GetCurrent>(fn);
        fn = nullptr;
        if (cudaGetDriverEntryPoint("cuCtxGetId", &fn, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_id = reinterpret_cast<GetId>(fn);
    });
    void *ctx = nullptr;
    unsigned long long id = 0;
    if (get_current && get_id && get_current(&ctx) == 0 && ctx && get_id(ctx, &id) == 0) return id;
    return 0;
}

// Device addresses of the two arrays on `device` (the current device), looked
// up once per device and context: a lookup is reused only while the context
// it was made in is still the current one.
bool noalloc_scratch(int device, NoAllocScratch &out) {
    static std::mutex mu;
    static NoAllocScratch cache[64];
    static unsigned long long context[64] = {};
    if (device < 0 || device >= 64) {
        set_error("device ordinal outside the no-allocation scratch table");
        return false;
    }
    const unsigned long long ctx = current_context_id();
    std::lock_guard<std::mutex> lock(mu);
    if (!ctx || context[device] != ctx) {
        void *q = nullptr, *xs = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&q, g_noalloc_q);
        if (e == cudaSuccess) e = cudaGetSymbolAddress(&xs, g_noalloc_xs);
        if (e != cudaSuccess || !q || !xs) {
            context[device] = 0;
            set_error(std::string("no-allocation scratch lookup failed: ") + cudaGetErrorString(e));
            return false;
        }
        cache[device].q = static_cast<int8_t *>(q);
        cache[device].xs = static_cast<float *>(xs);
        context[device] = ctx;
    }
    out = cache[device];
    return true;
}

}  // namespace
}  // namespace nb200

extern "C" int needle2_sdot_linear_device_noalloc(void *handle, const float *x, float *y, int batch, void *stream) {
    nb200::clear_error();
    auto *m = static_cast<Matrix *>(handle);
    if (!m || !m->sdot) { nb200::set_error("null or wrong-kind handle"); return -1; }
    if (batch < 0) { nb200::set_error("negative batch"); return -1; }
    if (batch == 0) return 0;
    const nb200::CQDevice &w = m->w;
    if ((size_t)batch * w.padded > nb200::kNoAllocActivationBytes ||
        (size_t)batch * w.groups > nb200::kNoAllocScales) {
        nb200::set_error("batch too large for the no-allocation scratch: batch * padded input must be <= 1048576 "
                         "and batch * groups <= 16384; use needle2_sdot_linear_device");
        return -1;
    }
    if (cudaSetDevice(m->device) != cudaSuccess) { nb200::set_error("cudaSetDevice failed"); return -1; }
    nb200::NoAllocScratch s;
    if (!nb200::noalloc_scratch(m->device, s)) return -1;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (!nb200::launch_quantize(w, x, batch, s.q, s.xs, st)) return -1;
    return nb200::launch_gemv_i8(w, s.q, s.xs, batch, y, w.out, nullptr, st) ? 0 : -1;
}

extern "C" int needle2_b200_set_f32_gemv(int kind) {
    const int previous = nb200::f32_gemv_kernel();
    if (kind < 0 || kind > 2) {
        nb200::set_error("FP32 GEMV kernel kind must be 0 (automatic), 1 (slot-per-lane kernel) or 2 (row-per-lane "
                         "kernel without the product table)");
        return -1;
    }
    nb200::set_f32_gemv_kernel(kind);
    return previous;
}
