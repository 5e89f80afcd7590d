// capi.cu - the extern "C" entry points declared in include/hynomas_b200.h.
//
// Each entry validates its arguments on the host (shapes, null pointers, enum values, the 16-byte
// alignment the vector/TMA paths rely on), checks once per device that it is a compute capability 10.0
// part, launches on the caller's stream and returns an hn_status. Errors never abort the process; the
// message is kept per calling thread for hn_last_error().
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <atomic>
#include <mutex>
#include <string>

#include <cmath>
#include <cuda.h>
#include <cudaTypedefs.h>

#include "../../include/hynomas_b200.h"
#include "hn_common.cuh"
#include "hn_kernels.h"

namespace hn {

static thread_local std::string t_last_error;

static int fail(int code, const char *fmt, ...) __attribute__((format(printf, 2, 3)));
static int fail(int code, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    t_last_error = buf;
    return code;
}

static int cuda_fail(cudaError_t e, const char *what) {
    return fail(HN_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

constexpr int MAX_DEV = HN_MAX_DEV;
static int g_sms[MAX_DEV];
static int g_arch_ok[MAX_DEV];  // 0 unknown, 1 ok, -1 not sm_100
static std::mutex g_mu;

static int current_device(int *dev) {
    cudaError_t e = cudaGetDevice(dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    if (*dev < 0 || *dev >= MAX_DEV) return fail(HN_ERR_ARG, "device index %d out of range", *dev);
    return HN_OK;
}

static int check_arch() {
    int dev;
    int rc = current_device(&dev);
    if (rc) return rc;
    if (g_arch_ok[dev] == 0) {
        std::lock_guard<std::mutex> lk(g_mu);
        int major = 0, minor = 0, sms = 0;
        cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
        cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        g_sms[dev] = sms;
        g_arch_ok[dev] = (major == 10 && minor == 0) ? 1 : -1;
        if (g_arch_ok[dev] < 0) t_last_error = "";
    }
    if (g_arch_ok[dev] < 0) {
        int major = 0, minor = 0;
        cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
        cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
        return fail(HN_ERR_ARCH, "device %d is sm_%d%d; this library runs on sm_100a (B200) only", dev, major, minor);
    }
    return HN_OK;
}

static std::atomic<int> g_gemm_sm_reserve{0};
int gemm_sm_reserve() { return g_gemm_sm_reserve.load(std::memory_order_relaxed); }

// stream -> error-word slot (slot 0: the NULL stream, and every stream once the table is full)
static cudaStream_t g_slot_stream[HN_ERR_SLOTS];
static int g_slots_used = 1;

int err_slot(cudaStream_t st) {
    if (st == nullptr) return 0;
    std::lock_guard<std::mutex> lk(g_mu);
    for (int i = 1; i < g_slots_used; ++i)
        if (g_slot_stream[i] == st) return i;
    if (g_slots_used == HN_ERR_SLOTS) return 0;
    g_slot_stream[g_slots_used] = st;
    return g_slots_used++;
}

int num_sms() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= MAX_DEV) return 148;
    if (g_sms[dev] == 0) {
        int sms = 0;
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        g_sms[dev] = sms > 0 ? sms : 148;
    }
    return g_sms[dev];
}

static inline bool al16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }
static inline bool al8(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 7) == 0; }
static inline int dsize(int dt) { return dt == HN_DTYPE_FP32 || dt == HN_DTYPE_INT32 ? 4 : 2; }

// A [rows, groups] scale tensor addressed as s[r * rs + g * gs] must not alias two entries: one stride
// must cover the whole extent of the other dimension (row-major: rs >= groups * gs; group-major:
// gs >= rows * rs).
static bool scale_strides_ok(int64_t rows, int64_t groups, int64_t rs, int64_t gs) {
    if (rows <= 1 && groups <= 1) return true;
    if (rows <= 1) return gs >= 1;
    if (groups <= 1) return rs >= 1;
    if (rs < 1 || gs < 1) return false;
    return rs >= groups * gs || gs >= rows * rs;
}

// The device that owns `stream` made current for the duration of an entry point (the caller's current device
// is put back on exit), so a launch, the SM count and the architecture check all refer to the stream's
// device whichever device the calling thread had current. The NULL stream keeps the current device.
struct StreamDevice {
    int prev = -1;
    cudaError_t err = cudaSuccess;
    explicit StreamDevice(void *stream) {
        if (stream == nullptr) return;
        int want = 0, cur = 0;
        err = cudaStreamGetDevice(static_cast<cudaStream_t>(stream), &want);
        if (err != cudaSuccess) return;
        err = cudaGetDevice(&cur);
        if (err != cudaSuccess || cur == want) return;
        err = cudaSetDevice(want);
        if (err == cudaSuccess) prev = cur;
    }
    ~StreamDevice() {
        if (prev >= 0) cudaSetDevice(prev);
    }
    StreamDevice(const StreamDevice &) = delete;
    StreamDevice &operator=(const StreamDevice &) = delete;
};

// The data must live on the launch device: the library enables no peer access, and a kernel handed another
// device's (or host) memory would fault. Checked on each call's main input before anything is launched.
static int check_pointer_device(const void *p, const char *what) {
    cudaPointerAttributes at;
    cudaError_t e = cudaPointerGetAttributes(&at, p);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return fail(HN_ERR_ARG, "%s: %p is not memory CUDA knows (%s)", what, p, cudaGetErrorString(e));
    }
    int dev = -1;
    e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    if (at.type == cudaMemoryTypeManaged) return HN_OK;
    if (at.type != cudaMemoryTypeDevice)
        return fail(HN_ERR_ARG, "%s: %p is not device memory", what, p);
    if (at.device != dev)
        return fail(HN_ERR_ARG, "%s: the data is on device %d but the launch device is %d (pass a stream of the "
                    "data's device, or make that device current for the NULL stream)", what, at.device, dev);
    return HN_OK;
}

static int launched(cudaError_t e, const char *what) {
    if (e != cudaSuccess) return cuda_fail(e, what);
    t_last_error.clear();
    return HN_OK;
}

} // namespace hn

using namespace hn;

// the stream's device made current for the rest of the entry point, then the architecture check on it, and
// the check that the main input `ptr` lives on it
#define CHECK_DEVICE(ptr)                                                                   \
    StreamDevice _stream_device(stream);                                                    \
    if (_stream_device.err != cudaSuccess) return cuda_fail(_stream_device.err, "cudaStreamGetDevice"); \
    do {                                                                                    \
        int _rc = check_arch();                                                             \
        if (_rc == HN_OK) _rc = check_pointer_device((ptr), __func__);                      \
        if (_rc != HN_OK) return _rc;                                                       \
    } while (0)
#define CHECK_ARCH()                                                                        \
    StreamDevice _stream_device(stream);                                                    \
    if (_stream_device.err != cudaSuccess) return cuda_fail(_stream_device.err, "cudaStreamGetDevice"); \
    do {                                                                                    \
        int _rc = check_arch();                                                             \
        if (_rc != HN_OK) return _rc;                                                       \
    } while (0)
#define REQUIRE(cond, code, ...)                      \
    do {                                              \
        if (!(cond)) return fail((code), __VA_ARGS__); \
    } while (0)

extern "C" {

const char *hn_last_error(void) { return t_last_error.c_str(); }

int hn_abi_version(void) { return HN_ABI_VERSION; }

int hn_set_gemm_sm_reserve(int n) {
    if (n < 0 || n > 64) return fail(HN_ERR_ARG, "hn_set_gemm_sm_reserve: n must be in [0, 64]");
    hn::g_gemm_sm_reserve.store(n, std::memory_order_relaxed);
    return HN_OK;
}

int hn_get_gemm_sm_reserve(void) { return hn::gemm_sm_reserve(); }

int hn_num_sms(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
        cudaGetLastError();
        return 0;
    }
    return num_sms();
}

int hn_device_error(void *stream, int *code_host) {
    REQUIRE(code_host != nullptr, HN_ERR_ARG, "code_host is NULL");
    StreamDevice sd(stream);
    if (sd.err != cudaSuccess) return cuda_fail(sd.err, "cudaStreamGetDevice");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return cuda_fail(e, "cudaStreamSynchronize");
    int v = 0;
    e = read_and_clear_device_error(err_slot(st), &v);
    if (e != cudaSuccess) return cuda_fail(e, "reading the device error word");
    *code_host = v;
    if (v & HN_DEVERR_TIMEOUT) return fail(HN_ERR_TIMEOUT, "a device-side wait ran past its limit");
    t_last_error.clear();
    return HN_OK;
}

int hn_selftest_wait_timeout(uint32_t timeout_us, void *stream) {
    CHECK_ARCH();
    REQUIRE(timeout_us > 0 && timeout_us <= 2000000u, HN_ERR_ARG, "timeout_us must be in (0, 2e6]");
    return launched(launch_wait_selftest(timeout_us, static_cast<cudaStream_t>(stream)), "wait self-test launch");
}

int hn_quant_act(const void *x, int64_t ldx, int x_dtype, int64_t M, int64_t K, int kind, int flags, void *q,
                 int64_t ldq, float *s, int64_t s_rs, int64_t s_gs, void *stream) {
    REQUIRE(x && q && s, HN_ERR_ARG, "hn_quant_act: null pointer");
    REQUIRE((flags & ~(HN_QUANT_PER_ROW | HN_QUANT_ROUND_HALF_EVEN)) == 0, HN_ERR_ARG, "hn_quant_act: unknown flags %d", flags);
    REQUIRE(!(flags & HN_QUANT_ROUND_HALF_EVEN) || kind == HN_KIND_INT8, HN_ERR_ARG,
            "hn_quant_act: round-half-even applies to int8 codes (e4m3 always rounds to nearest even)");
    const bool per_row = (flags & HN_QUANT_PER_ROW) != 0;
    REQUIRE(x_dtype == HN_DTYPE_BF16 || x_dtype == HN_DTYPE_FP16 || x_dtype == HN_DTYPE_FP32, HN_ERR_ARG,
            "hn_quant_act: x_dtype %d not bf16/fp16/fp32", x_dtype);
    REQUIRE(kind == HN_KIND_INT8 || kind == HN_KIND_FP8E4M3, HN_ERR_ARG, "hn_quant_act: unknown kind %d", kind);
    REQUIRE(M >= 0 && K > 0 && K % 128 == 0, HN_ERR_SHAPE, "hn_quant_act: need K %% 128 == 0 (M=%lld K=%lld)",
            (long long)M, (long long)K);
    REQUIRE(ldx >= K && ldq >= K, HN_ERR_SHAPE, "hn_quant_act: leading dimension too small");
    REQUIRE(scale_strides_ok(M, per_row ? 1 : K / 128, s_rs, s_gs), HN_ERR_SHAPE,
            "hn_quant_act: scale strides (%lld, %lld) overlap", (long long)s_rs, (long long)s_gs);
    REQUIRE(M <= 0x7fffffffLL, HN_ERR_SHAPE, "hn_quant_act: M too large");
    REQUIRE(al16(x) && (ldx * dsize(x_dtype)) % 16 == 0 && al16(q) && ldq % 16 == 0, HN_ERR_ALIGN,
            "hn_quant_act: x/q must be 16-byte aligned with 16-byte row pitch");
    if (M == 0) return HN_OK;
    CHECK_DEVICE(x);
    return launched(launch_quant_act(x, ldx, x_dtype, M, K, kind, flags, q, ldq, s, s_rs, s_gs, (cudaStream_t)stream),
                    "hn_quant_act launch");
}

int hn_block_gemm(const void *qa, int64_t lda, const float *sa, int64_t sa_rs, int64_t sa_gs, int sa_mode,
                  const void *qw, int64_t ldw, const float *sw, int64_t sw_rs, int64_t sw_gs, int sw_mode,
                  const void *bias, int bias_dtype, void *out, int64_t ldo, int out_dtype, float *qs, int64_t qs_rs,
                  int64_t qs_gs, int64_t M, int64_t N, int64_t K, int kind, int epilogue, void *stream) {
    REQUIRE(qa && sa && qw && sw && out, HN_ERR_ARG, "hn_block_gemm: null pointer");
    REQUIRE(kind == HN_KIND_INT8 || kind == HN_KIND_FP8E4M3, HN_ERR_ARG, "hn_block_gemm: unknown kind %d", kind);
    REQUIRE(sa_mode == HN_SCALE_GROUP || sa_mode == HN_SCALE_ROW, HN_ERR_ARG, "hn_block_gemm: bad sa_mode %d", sa_mode);
    REQUIRE(sw_mode >= HN_SCALE_GROUP && sw_mode <= HN_SCALE_BLOCK, HN_ERR_ARG, "hn_block_gemm: bad sw_mode %d", sw_mode);
    REQUIRE(epilogue >= HN_EPI_NONE && epilogue <= HN_EPI_GELU_QUANT, HN_ERR_ARG, "hn_block_gemm: bad epilogue %d", epilogue);
    REQUIRE(M >= 0 && N > 0 && K > 0 && K % 128 == 0, HN_ERR_SHAPE,
            "hn_block_gemm: need K %% 128 == 0, N > 0 (M=%lld N=%lld K=%lld)", (long long)M, (long long)N, (long long)K);
    REQUIRE(M < (1LL << 31) && N < (1LL << 31) && K < (1LL << 31), HN_ERR_SHAPE, "hn_block_gemm: dimension too large");
    // both scales per row: the tensor core sums all of K in one int32 accumulator, |sum| <= K * 128 * 128
    REQUIRE(!(kind == HN_KIND_INT8 && sa_mode == HN_SCALE_ROW && sw_mode == HN_SCALE_ROW) || K <= HN_ROW_MODE_MAX_K,
            HN_ERR_SHAPE, "hn_block_gemm: int8 with per-row scales on both sides needs K <= %d (int32 accumulator; K=%lld)",
            HN_ROW_MODE_MAX_K, (long long)K);
    REQUIRE(lda >= K && ldw >= K && ldo >= N, HN_ERR_SHAPE, "hn_block_gemm: leading dimension too small");
    REQUIRE(sa_mode != HN_SCALE_GROUP || scale_strides_ok(M, K / 128, sa_rs, sa_gs), HN_ERR_SHAPE,
            "hn_block_gemm: activation scale strides overlap");
    REQUIRE(sw_mode != HN_SCALE_GROUP || scale_strides_ok(N, K / 128, sw_rs, sw_gs), HN_ERR_SHAPE,
            "hn_block_gemm: weight scale strides overlap");
    REQUIRE(sw_mode != HN_SCALE_BLOCK || scale_strides_ok(cdiv(N, 128), K / 128, sw_rs, sw_gs), HN_ERR_SHAPE,
            "hn_block_gemm: weight block scale strides overlap");
    REQUIRE(sa_mode != HN_SCALE_ROW || sa_rs >= 1, HN_ERR_SHAPE, "hn_block_gemm: sa_rs < 1");
    REQUIRE(sw_mode != HN_SCALE_ROW || sw_rs >= 1, HN_ERR_SHAPE, "hn_block_gemm: sw_rs < 1");
    REQUIRE(al16(qa) && al16(qw) && lda % 16 == 0 && ldw % 16 == 0, HN_ERR_ALIGN,
            "hn_block_gemm: qa/qw must be 16-byte aligned with row pitch a multiple of 16");
    if (epilogue == HN_EPI_GELU_QUANT) {
        REQUIRE(qs != nullptr, HN_ERR_ARG, "hn_block_gemm: gelu_quant needs qs");
        REQUIRE(N % 128 == 0, HN_ERR_SHAPE, "hn_block_gemm: gelu_quant needs N %% 128 == 0");
        REQUIRE(scale_strides_ok(M, N / 128, qs_rs, qs_gs), HN_ERR_SHAPE, "hn_block_gemm: qs strides overlap");
        REQUIRE(al16(out) && ldo % 16 == 0, HN_ERR_ALIGN, "hn_block_gemm: int8 output must be 16-byte aligned");
    } else if (epilogue == HN_EPI_GELU) {
        REQUIRE(out_dtype == HN_DTYPE_BF16, HN_ERR_UNSUPPORTED, "hn_block_gemm: gelu output is bf16");
    } else {
        REQUIRE(out_dtype >= HN_DTYPE_BF16 && out_dtype <= HN_DTYPE_INT32, HN_ERR_ARG, "hn_block_gemm: bad out_dtype %d", out_dtype);
    }
    if (out_dtype == HN_DTYPE_INT32)
        REQUIRE(kind == HN_KIND_INT8 && sa_mode == HN_SCALE_ROW && sw_mode == HN_SCALE_ROW && bias == nullptr &&
                    epilogue == HN_EPI_NONE,
                HN_ERR_UNSUPPORTED, "hn_block_gemm: int32 output is the raw int8 accumulator (row scales, no bias)");
    if (bias) REQUIRE(bias_dtype == HN_DTYPE_BF16 || bias_dtype == HN_DTYPE_FP16 || bias_dtype == HN_DTYPE_FP32,
                      HN_ERR_ARG, "hn_block_gemm: bad bias dtype %d", bias_dtype);
    // the epilogue reads the bias 8 columns at a time with 16-byte loads wherever 8 columns are in range
    if (bias) REQUIRE(al16(bias), HN_ERR_ALIGN, "hn_block_gemm: bias must be 16-byte aligned");
    if (M == 0) return HN_OK;
    CHECK_DEVICE(qa);
    GemmArgs a;
    a.qa = qa; a.lda = lda; a.sa = sa; a.sa_rs = sa_rs; a.sa_gs = sa_gs; a.sa_mode = sa_mode;
    a.qw = qw; a.ldw = ldw; a.sw = sw; a.sw_rs = sw_rs; a.sw_gs = sw_gs; a.sw_mode = sw_mode;
    a.bias = bias; a.bias_dtype = bias_dtype;
    a.out = out; a.ldo = ldo; a.out_dtype = out_dtype; a.qs = qs; a.qs_rs = qs_rs; a.qs_gs = qs_gs;
    a.M = M; a.N = N; a.K = K; a.kind = kind; a.epilogue = epilogue;
    a.sm_reserve = gemm_sm_reserve();
    const char *msg = nullptr;
    cudaError_t e = launch_block_gemm(a, (cudaStream_t)stream, &msg);
    if (e != cudaSuccess && msg) return fail(HN_ERR_ALIGN, "hn_block_gemm: %s", msg);
    return launched(e, "hn_block_gemm launch");
}

static int ln_common(const void *x, const void *shift, const void *scale, int64_t B, int64_t L, int64_t D, int quant,
                     const char *name) {
    REQUIRE(x && shift && scale, HN_ERR_ARG, "%s: null pointer", name);
    REQUIRE(B > 0 && L >= 0 && D > 0 && D <= 16384, HN_ERR_SHAPE, "%s: bad shape B=%lld L=%lld D=%lld", name,
            (long long)B, (long long)L, (long long)D);
    REQUIRE(quant ? D % 128 == 0 : D % 16 == 0, HN_ERR_SHAPE, "%s: D %% %d != 0", name, quant ? 128 : 16);
    REQUIRE(B * L < (1LL << 31), HN_ERR_SHAPE, "%s: too many rows", name);
    REQUIRE(al16(x) && al16(shift) && al16(scale), HN_ERR_ALIGN, "%s: inputs must be 16-byte aligned", name);
    return HN_OK;
}

int hn_adaln_quant(const void *x, const void *shift, const void *scale, int64_t B, int64_t L, int64_t D, float eps,
                   int8_t *q, float *s, int64_t s_rs, int64_t s_gs, void *stream) {
    int rc = ln_common(x, shift, scale, B, L, D, 1, "hn_adaln_quant");
    if (rc) return rc;
    REQUIRE(q && s && al16(q), HN_ERR_ARG, "hn_adaln_quant: null or misaligned output");
    REQUIRE(scale_strides_ok(B * L, D / 128, s_rs, s_gs), HN_ERR_SHAPE, "hn_adaln_quant: scale strides overlap");
    if (L == 0) return HN_OK;
    CHECK_DEVICE(x);
    return launched(launch_ln_row(1, x, nullptr, nullptr, shift, scale, B, L, D, eps, nullptr, q, s, s_rs, s_gs,
                                  (cudaStream_t)stream),
                    "hn_adaln_quant launch");
}

int hn_adaln(const void *x, const void *shift, const void *scale, int64_t B, int64_t L, int64_t D, float eps, void *y,
             void *stream) {
    int rc = ln_common(x, shift, scale, B, L, D, 0, "hn_adaln");
    if (rc) return rc;
    REQUIRE(y && al16(y), HN_ERR_ARG, "hn_adaln: null or misaligned output");
    if (L == 0) return HN_OK;
    CHECK_DEVICE(x);
    return launched(launch_ln_row(0, x, nullptr, nullptr, shift, scale, B, L, D, eps, y, nullptr, nullptr, 0, 0,
                                  (cudaStream_t)stream),
                    "hn_adaln launch");
}

int hn_gated_residual_adaln_quant(const void *x, const void *y, const void *gate, const void *shift, const void *scale,
                                  int64_t B, int64_t L, int64_t D, float eps, void *out, int8_t *q, float *s,
                                  int64_t s_rs, int64_t s_gs, void *stream) {
    int rc = ln_common(x, shift, scale, B, L, D, 1, "hn_gated_residual_adaln_quant");
    if (rc) return rc;
    REQUIRE(y && gate && out && q && s, HN_ERR_ARG, "hn_gated_residual_adaln_quant: null pointer");
    REQUIRE(al16(y) && al16(gate) && al16(out) && al16(q), HN_ERR_ALIGN,
            "hn_gated_residual_adaln_quant: buffers must be 16-byte aligned");
    REQUIRE(scale_strides_ok(B * L, D / 128, s_rs, s_gs), HN_ERR_SHAPE,
            "hn_gated_residual_adaln_quant: scale strides overlap");
    if (L == 0) return HN_OK;
    CHECK_DEVICE(x);
    return launched(launch_ln_row(2, x, y, gate, shift, scale, B, L, D, eps, out, q, s, s_rs, s_gs, (cudaStream_t)stream),
                    "hn_gated_residual_adaln_quant launch");
}

int hn_gated_residual(const void *x, const void *y, const void *gate, int64_t B, int64_t L, int64_t D, void *out,
                      void *stream) {
    REQUIRE(x && y && gate && out, HN_ERR_ARG, "hn_gated_residual: null pointer");
    REQUIRE(B > 0 && L >= 0 && D > 0 && D % 8 == 0, HN_ERR_SHAPE, "hn_gated_residual: need D %% 8 == 0");
    REQUIRE(al16(x) && al16(y) && al16(gate) && al16(out), HN_ERR_ALIGN, "hn_gated_residual: buffers must be 16-byte aligned");
    if (L == 0) return HN_OK;
    CHECK_DEVICE(x);
    return launched(launch_gated_residual(x, y, gate, B, L, D, out, (cudaStream_t)stream), "hn_gated_residual launch");
}

static int qk_common(const void *x, int64_t row_stride, const void *w, const float *cos, const float *sin, int64_t B,
                     int64_t L, int64_t H, int64_t D, const void *y) {
    REQUIRE(x && w && y, HN_ERR_ARG, "hn_qk_norm_rope: null pointer");
    REQUIRE((cos == nullptr) == (sin == nullptr), HN_ERR_ARG, "hn_qk_norm_rope: cos and sin must both be given or both NULL");
    REQUIRE(D == 128, HN_ERR_UNSUPPORTED, "hn_qk_norm_rope: head dim %lld (kernels are built for 128)", (long long)D);
    REQUIRE(B > 0 && L >= 0 && H > 0 && row_stride >= H * D, HN_ERR_SHAPE, "hn_qk_norm_rope: bad shape/stride");
    REQUIRE(al16(x) && row_stride % 8 == 0 && al16(w) && al16(y), HN_ERR_ALIGN,
            "hn_qk_norm_rope: x/w/y must be 16-byte aligned with a row stride that is a multiple of 8");
    REQUIRE(cos == nullptr || (al16(cos) && al16(sin)), HN_ERR_ALIGN, "hn_qk_norm_rope: cos/sin must be 16-byte aligned");
    return HN_OK;
}

int hn_qk_norm_rope(const void *x, int64_t row_stride, const void *weight, const float *cos, const float *sin,
                    int64_t B, int64_t L, int64_t H, int64_t D, float eps, void *y, void *stream) {
    int rc = qk_common(x, row_stride, weight, cos, sin, B, L, H, D, y);
    if (rc) return rc;
    if (L == 0) return HN_OK;
    CHECK_DEVICE(x);
    return launched(launch_qk_norm_rope(1, x, nullptr, row_stride, weight, nullptr, cos, sin, B, L, H, eps, y, nullptr,
                                        nullptr, nullptr, (cudaStream_t)stream),
                    "hn_qk_norm_rope launch");
}

int hn_qk_norm_rope_kv(const void *x, int64_t row_stride, const void *weight, const float *cos, const float *sin,
                       int64_t B, int64_t L, int64_t H, int64_t D, float eps, void *y, int8_t *q, float *s,
                       void *stream) {
    int rc = qk_common(x, row_stride, weight, cos, sin, B, L, H, D, y);
    if (rc) return rc;
    REQUIRE(q && s, HN_ERR_ARG, "hn_qk_norm_rope_kv: null pointer");
    REQUIRE(al16(q) && (reinterpret_cast<uintptr_t>(s) & 3) == 0, HN_ERR_ALIGN, "hn_qk_norm_rope_kv: misaligned buffer");
    if (L == 0) return HN_OK;
    CHECK_DEVICE(x);
    return launched(launch_qk_norm_rope(1, x, nullptr, row_stride, weight, nullptr, cos, sin, B, L, H, eps, y, nullptr,
                                        q, s, (cudaStream_t)stream),
                    "hn_qk_norm_rope_kv launch");
}

int hn_qk_norm_rope2(const void *xq, const void *xk, int64_t row_stride, const void *wq, const void *wk,
                     const float *cos, const float *sin, int64_t B, int64_t L, int64_t H, int64_t D, float eps,
                     void *yq, void *yk, void *stream) {
    int rc = qk_common(xq, row_stride, wq, cos, sin, B, L, H, D, yq);
    if (rc) return rc;
    rc = qk_common(xk, row_stride, wk, cos, sin, B, L, H, D, yk);
    if (rc) return rc;
    if (L == 0) return HN_OK;
    CHECK_DEVICE(xq);
    return launched(launch_qk_norm_rope(2, xq, xk, row_stride, wq, wk, cos, sin, B, L, H, eps, yq, yk, nullptr, nullptr,
                                        (cudaStream_t)stream),
                    "hn_qk_norm_rope2 launch");
}

int hn_pixelumm_qk(const void *x, int64_t row_stride, const void *weight_t, const void *weight_hw, const float *cos,
                   const float *sin, int64_t N, int64_t H, int64_t D, float eps, void *y, void *stream) {
    REQUIRE(x && weight_t && weight_hw && cos && sin && y, HN_ERR_ARG, "hn_pixelumm_qk: null pointer");
    REQUIRE(D == 128, HN_ERR_UNSUPPORTED, "hn_pixelumm_qk: head dim %lld (kernels are built for 128)", (long long)D);
    REQUIRE(N >= 0 && H > 0 && row_stride >= H * D, HN_ERR_SHAPE, "hn_pixelumm_qk: bad shape/stride");
    REQUIRE(al8(x) && row_stride % 4 == 0 && al8(weight_t) && al8(weight_hw) && al16(cos) && al16(sin) && al8(y),
            HN_ERR_ALIGN, "hn_pixelumm_qk: misaligned buffer");
    if (N == 0) return HN_OK;
    CHECK_DEVICE(x);
    return launched(launch_pixelumm_qk(x, row_stride, weight_t, weight_hw, cos, sin, N, H, eps, y, (cudaStream_t)stream),
                    "hn_pixelumm_qk launch");
}

int hn_quantize_kv(const void *x, int64_t rows, int64_t D, int8_t *q, float *s, void *stream) {
    REQUIRE(D > 0 && D % 128 == 0, HN_ERR_SHAPE, "hn_quantize_kv: need D %% 128 == 0");
    return hn_quant_act(x, D, HN_DTYPE_BF16, rows, D, HN_KIND_INT8, D == 128 ? 0 : 1, q, D, s, 1, 1, stream);
}

int hn_dequantize_kv(const int8_t *q, const float *s, int64_t rows, int64_t D, void *y, void *stream) {
    REQUIRE(q && s && y, HN_ERR_ARG, "hn_dequantize_kv: null pointer");
    REQUIRE(rows >= 0 && D > 0 && D % 16 == 0, HN_ERR_SHAPE, "hn_dequantize_kv: need D %% 16 == 0 (D=%lld)", (long long)D);
    REQUIRE(al16(q) && al16(y) && (reinterpret_cast<uintptr_t>(s) & 3) == 0, HN_ERR_ALIGN,
            "hn_dequantize_kv: misaligned buffer");
    if (rows == 0) return HN_OK;
    CHECK_DEVICE(q);
    return launched(launch_dequant_kv(q, s, rows, D, y, (cudaStream_t)stream), "hn_dequantize_kv launch");
}

int hn_rmsnorm_quant(const void *x, int64_t ldx, const void *weight, int64_t rows, int64_t D, float eps, int kind,
                     void *q, int64_t ldq, float *s, int64_t s_rs, int64_t s_gs, void *stream) {
    REQUIRE(x && weight && q && s, HN_ERR_ARG, "hn_rmsnorm_quant: null pointer");
    REQUIRE(kind == HN_KIND_INT8 || kind == HN_KIND_FP8E4M3, HN_ERR_ARG, "hn_rmsnorm_quant: unknown kind %d", kind);
    REQUIRE(rows >= 0 && D > 0 && D % 128 == 0 && D <= 16384, HN_ERR_SHAPE,
            "hn_rmsnorm_quant: need D %% 128 == 0 and D <= 16384 (D=%lld)", (long long)D);
    REQUIRE(rows < (1LL << 31) && ldx >= D && ldq >= D, HN_ERR_SHAPE, "hn_rmsnorm_quant: bad rows or leading dimension");
    REQUIRE(scale_strides_ok(rows, D / 128, s_rs, s_gs), HN_ERR_SHAPE, "hn_rmsnorm_quant: scale strides overlap");
    REQUIRE(al16(x) && ldx % 8 == 0 && al16(weight) && al16(q) && ldq % 16 == 0, HN_ERR_ALIGN,
            "hn_rmsnorm_quant: x/weight/q must be 16-byte aligned with 16-byte row pitches");
    if (rows == 0) return HN_OK;
    CHECK_DEVICE(x);
    return launched(launch_rmsnorm_quant(x, ldx, weight, rows, D, eps, kind, q, ldq, s, s_rs, s_gs, (cudaStream_t)stream),
                    "hn_rmsnorm_quant launch");
}

int hn_silu_mul_quant(const void *g, int64_t ldg, const void *u, int64_t ldu, int64_t rows, int64_t I, int kind,
                      void *q, int64_t ldq, float *s, int64_t s_rs, int64_t s_gs, void *stream) {
    REQUIRE(g && u && q && s, HN_ERR_ARG, "hn_silu_mul_quant: null pointer");
    REQUIRE(kind == HN_KIND_INT8 || kind == HN_KIND_FP8E4M3, HN_ERR_ARG, "hn_silu_mul_quant: unknown kind %d", kind);
    REQUIRE(rows >= 0 && I > 0 && I % 128 == 0, HN_ERR_SHAPE, "hn_silu_mul_quant: need I %% 128 == 0 (I=%lld)", (long long)I);
    REQUIRE(ldg >= I && ldu >= I && ldq >= I, HN_ERR_SHAPE, "hn_silu_mul_quant: leading dimension too small");
    REQUIRE(scale_strides_ok(rows, I / 128, s_rs, s_gs), HN_ERR_SHAPE, "hn_silu_mul_quant: scale strides overlap");
    REQUIRE(al16(g) && al16(u) && ldg % 8 == 0 && ldu % 8 == 0 && al16(q) && ldq % 16 == 0, HN_ERR_ALIGN,
            "hn_silu_mul_quant: g/u/q must be 16-byte aligned with 16-byte row pitches");
    if (rows == 0) return HN_OK;
    CHECK_DEVICE(g);
    return launched(launch_silu_mul_quant(g, ldg, u, ldu, rows, I, kind, q, ldq, s, s_rs, s_gs, (cudaStream_t)stream),
                    "hn_silu_mul_quant launch");
}

int hn_quantize_fp8_block(const void *w, int w_dtype, int64_t N, int64_t K, void *q, float *s, void *stream) {
    REQUIRE(w && q && s, HN_ERR_ARG, "hn_quantize_fp8_block: null pointer");
    REQUIRE(w_dtype == HN_DTYPE_FP32 || w_dtype == HN_DTYPE_BF16, HN_ERR_ARG,
            "hn_quantize_fp8_block: w_dtype %d not fp32/bf16", w_dtype);
    REQUIRE(N >= 0 && K >= 0 && N % 128 == 0 && K % 128 == 0, HN_ERR_SHAPE,
            "hn_quantize_fp8_block: need N %% 128 == 0 and K %% 128 == 0 (N=%lld K=%lld)", (long long)N, (long long)K);
    REQUIRE(N / 128 <= 65535 && K / 128 <= 0x7fffffffLL, HN_ERR_SHAPE, "hn_quantize_fp8_block: too large");
    REQUIRE(al16(w) && al16(q) && (reinterpret_cast<uintptr_t>(s) & 3) == 0, HN_ERR_ALIGN, "hn_quantize_fp8_block: misaligned buffer");
    if (N == 0 || K == 0) return HN_OK;
    CHECK_DEVICE(w);
    return launched(launch_quant_fp8_block(w, w_dtype, N, K, q, s, (cudaStream_t)stream), "hn_quantize_fp8_block launch");
}

int hn_attention(const void *q, int64_t q_rs, int64_t q_hs, int64_t q_bs, const void *k, int64_t k_rs, int64_t k_hs,
                 int64_t k_bs, const void *v, int64_t v_rs, int64_t v_hs, int64_t v_bs, int64_t B, int64_t Lq,
                 int64_t Lk, int64_t H, int64_t D, float scale, void *out, int64_t o_rs, int64_t o_hs, int64_t o_bs,
                 int8_t *q8, float *s8, void *stream) {
    REQUIRE(q && k && v, HN_ERR_ARG, "hn_attention: null q/k/v");
    REQUIRE(out != nullptr || q8 != nullptr, HN_ERR_ARG, "hn_attention: no output (out and q8 both null)");
    REQUIRE((q8 == nullptr) == (s8 == nullptr), HN_ERR_ARG, "hn_attention: q8 and s8 go together");
    REQUIRE(D == 128, HN_ERR_UNSUPPORTED, "hn_attention: head dim %lld (128 supported)", (long long)D);
    REQUIRE(B >= 1 && H >= 1 && Lq >= 1 && Lk >= 1, HN_ERR_SHAPE, "hn_attention: empty shape B=%lld H=%lld Lq=%lld Lk=%lld",
            (long long)B, (long long)H, (long long)Lq, (long long)Lk);
    REQUIRE(B <= 65535 && H <= 65535 && Lq < (1LL << 31) && Lk < (1LL << 31) && B * Lq < (1LL << 31), HN_ERR_SHAPE,
            "hn_attention: too large");
    REQUIRE(std::isfinite(scale) && scale > 0.0f, HN_ERR_ARG, "hn_attention: scale must be positive and finite");
    const int64_t st_in[9] = {q_rs, q_hs, q_bs, k_rs, k_hs, k_bs, v_rs, v_hs, v_bs};
    for (int i = 0; i < 9; ++i)
        REQUIRE(st_in[i] >= 0 && st_in[i] % 8 == 0 && st_in[i] < (1LL << 38), HN_ERR_ALIGN,
                "hn_attention: input strides must be non-negative multiples of 8 elements");
    REQUIRE(al16(q) && al16(k) && al16(v), HN_ERR_ALIGN, "hn_attention: q/k/v must be 16-byte aligned");
    if (out != nullptr)
        REQUIRE(al16(out) && o_rs >= 0 && o_hs >= 0 && o_bs >= 0 && o_rs % 8 == 0 && o_hs % 8 == 0 && o_bs % 8 == 0,
                HN_ERR_ALIGN, "hn_attention: out must be 16-byte aligned with strides multiples of 8 elements");
    if (q8 != nullptr)
        REQUIRE(reinterpret_cast<uintptr_t>(q8) % 8 == 0 && reinterpret_cast<uintptr_t>(s8) % 4 == 0, HN_ERR_ALIGN,
                "hn_attention: q8 must be 8-byte and s8 4-byte aligned");
    CHECK_DEVICE(q);
    AttnArgs a;
    a.q = q; a.k = k; a.v = v;
    a.q_rs = q_rs; a.q_hs = q_hs; a.q_bs = q_bs; a.k_rs = k_rs; a.k_hs = k_hs; a.k_bs = k_bs;
    a.v_rs = v_rs; a.v_hs = v_hs; a.v_bs = v_bs;
    a.B = B; a.Lq = Lq; a.Lk = Lk; a.H = H; a.scale = scale;
    a.out = out; a.o_rs = o_rs; a.o_hs = o_hs; a.o_bs = o_bs; a.q8 = q8; a.s8 = s8;
    const char *msg = nullptr;
    cudaError_t e = launch_attention(a, (cudaStream_t)stream, &msg);
    if (e != cudaSuccess && msg) return fail(HN_ERR_ALIGN, "hn_attention: %s", msg);
    return launched(e, "hn_attention launch");
}

int hn_attn_merge(const void *const *parts, const float *const *lses, int64_t n, int64_t o_bs, int64_t o_qs,
                  int64_t o_hs, int64_t l_bs, int64_t l_hs, int64_t l_qs, int64_t B, int64_t Lq, int64_t H, int64_t D,
                  void *out, int64_t out_bs, int64_t out_qs, int64_t out_hs, int8_t *q8, float *s8, void *stream) {
    REQUIRE(parts && lses, HN_ERR_ARG, "hn_attn_merge: null piece arrays");
    REQUIRE(n >= 1 && n <= 16, HN_ERR_SHAPE, "hn_attn_merge: %lld pieces (1 to 16)", (long long)n);
    REQUIRE(out != nullptr || q8 != nullptr, HN_ERR_ARG, "hn_attn_merge: no output");
    REQUIRE((q8 == nullptr) == (s8 == nullptr), HN_ERR_ARG, "hn_attn_merge: q8 and s8 go together");
    REQUIRE(D == 128, HN_ERR_UNSUPPORTED, "hn_attn_merge: head dim %lld (128 supported)", (long long)D);
    REQUIRE(B >= 1 && Lq >= 0 && H >= 1 && B * Lq * H < (1LL << 40) && B * Lq < (1LL << 31), HN_ERR_SHAPE,
            "hn_attn_merge: bad shape");
    for (int64_t i = 0; i < n; ++i) {
        REQUIRE(parts[i] && lses[i], HN_ERR_ARG, "hn_attn_merge: null piece %lld", (long long)i);
        REQUIRE(reinterpret_cast<uintptr_t>(parts[i]) % 8 == 0 && reinterpret_cast<uintptr_t>(lses[i]) % 4 == 0,
                HN_ERR_ALIGN, "hn_attn_merge: piece %lld misaligned", (long long)i);
    }
    REQUIRE(o_bs % 4 == 0 && o_qs % 4 == 0 && o_hs % 4 == 0 && o_bs >= 0 && o_qs >= 0 && o_hs >= 0, HN_ERR_ALIGN,
            "hn_attn_merge: piece strides must be non-negative multiples of 4 elements");
    REQUIRE(l_bs >= 0 && l_hs >= 0 && l_qs >= 0, HN_ERR_ARG, "hn_attn_merge: negative log-sum-exp stride");
    if (out != nullptr)
        REQUIRE(reinterpret_cast<uintptr_t>(out) % 8 == 0 && out_bs % 4 == 0 && out_qs % 4 == 0 && out_hs % 4 == 0 &&
                    out_bs >= 0 && out_qs >= 0 && out_hs >= 0,
                HN_ERR_ALIGN, "hn_attn_merge: out must be 8-byte aligned with strides multiples of 4 elements");
    if (q8 != nullptr)
        REQUIRE(reinterpret_cast<uintptr_t>(q8) % 4 == 0 && reinterpret_cast<uintptr_t>(s8) % 4 == 0, HN_ERR_ALIGN,
                "hn_attn_merge: q8 / s8 must be 4-byte aligned");
    if (Lq == 0) return HN_OK;
    CHECK_DEVICE(parts[0]);
    MergeArgs a;
    a.parts = parts; a.lses = lses; a.n = n;
    a.o_bs = o_bs; a.o_qs = o_qs; a.o_hs = o_hs; a.l_bs = l_bs; a.l_hs = l_hs; a.l_qs = l_qs;
    a.B = B; a.Lq = Lq; a.H = H;
    a.out = out; a.out_bs = out_bs; a.out_qs = out_qs; a.out_hs = out_hs; a.q8 = q8; a.s8 = s8;
    return launched(launch_attn_merge(a, (cudaStream_t)stream), "hn_attn_merge launch");
}

} // extern "C"

// ---------------------------------------------------------------------------------------------------
// Sequence-parallel K/V exchange over NVLink by the copy engines (host-side only: CUDA IPC mappings, an
// asynchronous peer copy, a 32-bit flag write the GPU's front end executes after the copy - no SM involved - and a
// one-warp bounded wait for the peers' flags). No reference counterpart: the reference runs one GPU.

namespace hn {

typedef CUresult(CUDAAPI *PfnWrite32)(CUstream, CUdeviceptr, cuuint32_t, unsigned int);
typedef CUresult(CUDAAPI *PfnAddrRange)(CUdeviceptr *, size_t *, CUdeviceptr);

template <typename F> static F driver_fn(const char *name) {
    void *ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion(name, &ptr, 12000, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    return reinterpret_cast<F>(ptr);
}

static int cu_fail(CUresult r, const char *what) {
    return fail(HN_ERR_CUDA, "%s failed (CUresult %d)", what, (int)r);
}

} // namespace hn

extern "C" {

int hn_ipc_export(const void *ptr, void *handle_host, int64_t *offset_host) {
    REQUIRE(ptr && handle_host && offset_host, HN_ERR_ARG, "hn_ipc_export: null pointer");
    static PfnAddrRange range = driver_fn<PfnAddrRange>("cuMemGetAddressRange");
    REQUIRE(range != nullptr, HN_ERR_CUDA, "hn_ipc_export: cuMemGetAddressRange unavailable");
    CUdeviceptr base = 0;
    size_t size = 0;
    CUresult r = range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr));
    if (r != CUDA_SUCCESS) return cu_fail(r, "cuMemGetAddressRange");
    cudaIpcMemHandle_t h;
    cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void *>(base));
    if (e != cudaSuccess) return cuda_fail(e, "cudaIpcGetMemHandle");
    memcpy(handle_host, &h, sizeof(h));
    *offset_host = (int64_t)(reinterpret_cast<CUdeviceptr>(ptr) - base);
    t_last_error.clear();
    return HN_OK;
}

int hn_ipc_import(const void *handle_host, void **base_host) {
    REQUIRE(handle_host && base_host, HN_ERR_ARG, "hn_ipc_import: null pointer");
    cudaIpcMemHandle_t h;
    memcpy(&h, handle_host, sizeof(h));
    void *base = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return cuda_fail(e, "cudaIpcOpenMemHandle");
    *base_host = base;
    t_last_error.clear();
    return HN_OK;
}

int hn_ipc_close(void *base) {
    REQUIRE(base != nullptr, HN_ERR_ARG, "hn_ipc_close: null pointer");
    cudaError_t e = cudaIpcCloseMemHandle(base);
    if (e != cudaSuccess) return cuda_fail(e, "cudaIpcCloseMemHandle");
    t_last_error.clear();
    return HN_OK;
}

int hn_peer_push(void *dst, const void *src, int64_t bytes, void *flag, uint32_t value, void *stream) {
    REQUIRE(dst && src && bytes >= 0, HN_ERR_ARG, "hn_peer_push: null pointer or negative size");
    static PfnWrite32 write32 = driver_fn<PfnWrite32>("cuStreamWriteValue32");
    REQUIRE(flag == nullptr || write32 != nullptr, HN_ERR_CUDA, "hn_peer_push: cuStreamWriteValue32 unavailable");
    StreamDevice sd(stream);
    if (sd.err != cudaSuccess) return cuda_fail(sd.err, "cudaStreamGetDevice");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (bytes > 0) {
        cudaError_t e = cudaMemcpyAsync(dst, src, (size_t)bytes, cudaMemcpyDeviceToDevice, st);
        if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyAsync (peer push)");
    }
    if (flag != nullptr) {
        // default flags: a memory fence precedes the write, so the copy above is visible before the flag
        CUresult r = write32(reinterpret_cast<CUstream>(st), reinterpret_cast<CUdeviceptr>(flag), value, 0);
        if (r != CUDA_SUCCESS) return cu_fail(r, "cuStreamWriteValue32");
    }
    t_last_error.clear();
    return HN_OK;
}

int hn_peer_push2d(void *dst, int64_t dpitch, const void *src, int64_t spitch, int64_t width, int64_t height,
                   void *flag, uint32_t value, void *stream) {
    REQUIRE(dst && src, HN_ERR_ARG, "hn_peer_push2d: null pointer");
    REQUIRE(width >= 0 && height >= 0 && dpitch >= width && spitch >= width, HN_ERR_SHAPE,
            "hn_peer_push2d: need 0 <= width <= pitches and height >= 0 (width=%lld dpitch=%lld spitch=%lld "
            "height=%lld)", (long long)width, (long long)dpitch, (long long)spitch, (long long)height);
    static PfnWrite32 write32 = driver_fn<PfnWrite32>("cuStreamWriteValue32");
    REQUIRE(flag == nullptr || write32 != nullptr, HN_ERR_CUDA, "hn_peer_push2d: cuStreamWriteValue32 unavailable");
    StreamDevice sd(stream);
    if (sd.err != cudaSuccess) return cuda_fail(sd.err, "cudaStreamGetDevice");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (width > 0 && height > 0) {
        cudaError_t e = cudaMemcpy2DAsync(dst, (size_t)dpitch, src, (size_t)spitch, (size_t)width, (size_t)height,
                                          cudaMemcpyDeviceToDevice, st);
        if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpy2DAsync (peer push)");
    }
    if (flag != nullptr) {
        // default flags: a memory fence precedes the write, so the rows above are visible before the flag
        CUresult r = write32(reinterpret_cast<CUstream>(st), reinterpret_cast<CUdeviceptr>(flag), value, 0);
        if (r != CUDA_SUCCESS) return cu_fail(r, "cuStreamWriteValue32");
    }
    t_last_error.clear();
    return HN_OK;
}

int hn_wait_flags(const int32_t *flags, int64_t groups, int64_t count, int64_t group_stride, int64_t skip,
                  uint32_t value, uint32_t timeout_us, void *stream) {
    REQUIRE(flags != nullptr, HN_ERR_ARG, "hn_wait_flags: null pointer");
    REQUIRE(groups >= 0 && count >= 0 && groups <= 1024 && count <= 1024 && groups * count <= 1024, HN_ERR_SHAPE,
            "hn_wait_flags: need 0 <= groups * count <= 1024 (groups=%lld count=%lld)", (long long)groups,
            (long long)count);
    REQUIRE(group_stride >= 0 && group_stride <= (1LL << 20), HN_ERR_SHAPE, "hn_wait_flags: group_stride out of range");
    REQUIRE(timeout_us > 0 && timeout_us <= 600000000u, HN_ERR_ARG, "hn_wait_flags: timeout_us must be in (0, 6e8]");
    REQUIRE(((uintptr_t)flags % 4) == 0, HN_ERR_ALIGN, "hn_wait_flags: flags must be 4-byte aligned");
    if (groups * count == 0) return HN_OK;
    CHECK_DEVICE(flags);
    return launched(launch_wait_flags(reinterpret_cast<const uint32_t *>(flags), (int)groups, (int)count,
                                      (int)group_stride, (int)(skip < 0 || skip >= count ? -1 : skip), value,
                                      timeout_us, static_cast<cudaStream_t>(stream)),
                    "hn_wait_flags launch");
}

} // extern "C"
