// C ABI for CQ matrices on B200: handle lifetime, host validation, staging
// and the error channel.  Mirrors the reference entry points of
// needle2/csrc/cq.cpp:342-371 and needle2/csrc/sdot.cpp:349-360; all
// arithmetic runs in the kernels of cq_kernels.cu.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <new>
#include <string>
#include <vector>

#include "../../include/needle2_b200.h"
#include "common.cuh"
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

struct Matrix {
    CQDevice w{};
    bool sdot = false;
    int device = 0;
    cudaStream_t stream = nullptr;
    uint8_t *d_packed = nullptr;
    uint16_t *d_norms = nullptr;
    Scratch<float> x, y, rot, xs;
    Scratch<int8_t> q;
    Scratch<int32_t> partials;
    Scratch<int64_t> ids;
    int prepared = 0;  // activation rows held in rot / q+xs by the last prepare

    ~Matrix() {
        cudaSetDevice(device);
        if (stream) cudaStreamSynchronize(stream);
        x.release(); y.release(); rot.release(); xs.release(); q.release(); partials.release(); ids.release();
        if (d_packed) cudaFree(d_packed);
        if (d_norms) cudaFree(d_norms);
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
    return m;
}

// Enqueue y = W x on `st` for device x[batch][in] -> y[batch][out].
bool run_linear_device(Matrix *m, const float *x, float *y, int batch, cudaStream_t st, int32_t *partials) {
    m->prepared = 0;
    if (batch <= 0) return true;
    const CQDevice &w = m->w;
    if (!m->sdot) {
        if (!m->rot.reserve((size_t)batch * w.padded)) return false;
        if (!launch_rotate(w, x, batch, m->rot.ptr, st)) return false;
        return launch_gemv_f32(w, m->rot.ptr, batch, y, w.out, st);
    }
    if (!m->q.reserve((size_t)batch * w.padded) || !m->xs.reserve((size_t)batch * w.groups)) return false;
    if (!launch_quantize(w, x, batch, m->q.ptr, m->xs.ptr, st)) return false;
    return launch_gemv_i8(w, m->q.ptr, m->xs.ptr, batch, y, w.out, partials, st);
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

void needle2_cq_linear_many(void *const *handles, int count, const float *x, float *const *ys, int threads,
                            int mode) {
    (void)mode;
    nb200::clear_error();
    for (int i = 0; i < count; ++i) {
        if (needle2_cq_linear_checked(handles[i], x, ys[i], 1)) return;
    }
    (void)threads;
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
    bool ok = sdot ? nb200::launch_gemv_i8(w, m->q.ptr, m->xs.ptr, batch, y, w.out, nullptr, st)
                   : nb200::launch_gemv_f32(w, m->rot.ptr, batch, y, w.out, st);
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

int needle2_cq_geometry(void *handle, int *g) {
    auto *m = static_cast<Matrix *>(handle);
    if (!m || !g) { nb200::set_error("null handle"); return -1; }
    g[0] = m->w.out; g[1] = m->w.in; g[2] = m->w.bits; g[3] = m->w.group; g[4] = m->w.padded; g[5] = m->w.groups;
    return 0;
}

}  // extern "C"
