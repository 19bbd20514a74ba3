// Library lifecycle, error reporting, device registry and stream/workspace state.
//
// Mirrors the reference's control surface (src/ecpu/src/core/ecpu.c:17-81 and
// src/ecpu/src/device/*.c) with the CUDA slot filled in: the reference registers a
// "cuda (reserved)" vtable whose init returns -1 (cuda_device.c:5-28); here that slot
// is a working B200 device and it is the default active device.
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <mutex>
#include <vector>

#include "common.cuh"

#define PILM_VERSION_STRING "0.1.0-b200"

namespace {

struct State {
    int initialized = 0;
    ecpu_config_t config{};
    char err[512] = {0};
    cudaStream_t stream = nullptr;
    int sync = -1;
    void *ws[pilm::kScratchSlots] = {};
    size_t ws_bytes[pilm::kScratchSlots] = {};
    int *ctr = nullptr;
    size_t ctr_n = 0;
    // Outgrown scratch and counter buffers.  CUDA graphs captured earlier still hold
    // their addresses, so they stay allocated until ecpu_shutdown.
    std::vector<void *> retired;
};

State g;
std::mutex g_mu;

// ---- device vtables (device/api.h:31-46) -------------------------------------------

void *cuda_alloc(size_t bytes, size_t alignment) {
    (void)alignment;  // cudaMalloc returns 256-byte aligned memory
    void *p = nullptr;
    if (cudaMalloc(&p, bytes ? bytes : 1) != cudaSuccess) return nullptr;
    return p;
}
void cuda_free(void *p) { cudaFree(p); }
void cuda_h2d(void *d, const void *s, size_t n) { cudaMemcpy(d, s, n, cudaMemcpyHostToDevice); }
void cuda_d2h(void *d, const void *s, size_t n) { cudaMemcpy(d, s, n, cudaMemcpyDeviceToHost); }
void cuda_d2d(void *d, const void *s, size_t n) { cudaMemcpy(d, s, n, cudaMemcpyDeviceToDevice); }
int cuda_sync() { return cudaDeviceSynchronize() == cudaSuccess ? 0 : -1; }
size_t cuda_total() {
    size_t f = 0, t = 0;
    cudaMemGetInfo(&f, &t);
    return t;
}
size_t cuda_freemem() {
    size_t f = 0, t = 0;
    cudaMemGetInfo(&f, &t);
    return f;
}
int cuda_init() {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) return -1;
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceProp p;
    if (cudaGetDeviceProperties(&p, dev) != cudaSuccess) return -1;
    if (p.major < 10) return -1;  // sm_100a kernels only
    return 0;
}
int cuda_shutdown() { return 0; }

void *host_alloc(size_t bytes, size_t alignment) {
    if (alignment < sizeof(void *)) alignment = sizeof(void *);
    void *p = nullptr;
    if (posix_memalign(&p, alignment, bytes ? bytes : 1) != 0) return nullptr;
    return p;
}
void host_free(void *p) { free(p); }
void host_copy(void *d, const void *s, size_t n) { memcpy(d, s, n); }
int host_sync() { return 0; }
size_t host_zero() { return 0; }
int host_init() { return 0; }

const edevice_vtable_t kCudaVtable = {
    "cuda (B200 sm_100a)", EDEV_CUDA, (uint64_t)(EDEV_CAP_BF16 | EDEV_CAP_F16 | EDEV_CAP_FP8),
    cuda_alloc, cuda_free, cuda_h2d, cuda_d2h, cuda_d2d, cuda_sync, cuda_total, cuda_freemem,
    cuda_init, cuda_shutdown,
};
const edevice_vtable_t kHostVtable = {
    "ecpu (host memory)", EDEV_ECPU, (uint64_t)EDEV_CAP_NONE,
    host_alloc, host_free, host_copy, host_copy, host_copy, host_sync, host_zero, host_zero,
    host_init, host_init,
};

edevice_vtable_t g_registry[EDEV_COUNT];
int g_inited[EDEV_COUNT];
edevice_t g_active = EDEV_CUDA;
int g_registered = 0;

void register_defaults() {
    if (g_registered) return;
    g_registry[EDEV_ECPU] = kHostVtable;
    g_registry[EDEV_CUDA] = kCudaVtable;
    g_registered = 1;
}

}  // namespace

namespace pilm {

cudaStream_t stream() { return g.stream; }

int sync_mode() {
    if (g.sync < 0) {
        const char *v = getenv("PILM_CUDA_SYNC");
        g.sync = (v && strcmp(v, "1") == 0) ? 1 : 0;
    }
    return g.sync;
}

// The library stream is being captured into a CUDA graph: synchronous mode then neither
// synchronizes nor reads back (either would invalidate the capture).
bool capturing() {
    cudaStreamCaptureStatus st = cudaStreamCaptureStatusNone;
    return cudaStreamIsCapturing(g.stream, &st) == cudaSuccess && st != cudaStreamCaptureStatusNone;
}

TensorMapEncodeTiledFn tensor_map_encoder() {
    static TensorMapEncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (TensorMapEncodeTiledFn)ptr;
    });
    return fn;
}

// Device allocations the library made for itself (scratch, counters, error words); the
// vtable's alloc, which the caller asks for, is not counted.
static unsigned long long g_lib_allocs = 0;

namespace {
constexpr int kMaxDevices = 64;
int *g_err_word[kMaxDevices];
int g_sms_of[kMaxDevices];
std::mutex g_dev_mu;

int current_device() {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return -1;
    return dev;
}
}  // namespace

// One error word per device, allocated on that device the first time a kernel there needs
// it (a kernel must not write another device's word).
int *device_error_word() {
    const int dev = current_device();
    if (dev < 0) return nullptr;
    std::lock_guard<std::mutex> lk(g_dev_mu);
    if (!g_err_word[dev]) {
        int *w = nullptr;
        if (cudaMalloc(&w, sizeof(int)) != cudaSuccess) return nullptr;
        ++g_lib_allocs;
        if (cudaMemset(w, 0, sizeof(int)) != cudaSuccess) {
            cudaFree(w);
            return nullptr;
        }
        g_err_word[dev] = w;
    }
    return g_err_word[dev];
}

int check_error_word_at(int *err, const char *what, const char *msg) {
    if (!sync_mode() || !err || capturing()) return ECPU_OK;
    int h = 0;
    cudaMemcpy(&h, err, sizeof(int), cudaMemcpyDeviceToHost);
    if (h) {
        cudaMemset(err, 0, sizeof(int));
        set_error("%s: %s", what, msg);
        return ECPU_ERR_KERNEL;
    }
    return ECPU_OK;
}

int check_error_word(const char *what, const char *msg) {
    return check_error_word_at(device_error_word(), what, msg);
}

// SM count of the current device (cached per device).
int num_sms() {
    const int dev = current_device();
    if (dev < 0) return 148;
    std::lock_guard<std::mutex> lk(g_dev_mu);
    if (g_sms_of[dev] <= 0) {
        int n = 0;
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        g_sms_of[dev] = n > 0 ? n : 148;
    }
    return g_sms_of[dev];
}

void set_error(const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g.err, sizeof(g.err), fmt, ap);
    va_end(ap);
}

// Scratch memory.  Each slot grows only when a request exceeds its current size;
// growing inside stream capture is refused (the caller sees NULL and returns
// ECPU_ERR_MEM), so graph capture must follow one eager call of the same shapes.
// An outgrown buffer is retired, not freed: a graph captured while it was current
// replays into it.  Each growth at least doubles the slot, so the retired buffers
// together stay smaller than the live one.
void *scratch(int slot, size_t bytes) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (slot < 0 || slot >= kScratchSlots) return nullptr;
    if (bytes <= g.ws_bytes[slot]) return g.ws[slot];
    cudaStreamCaptureStatus st = cudaStreamCaptureStatusNone;
    cudaStreamIsCapturing(g.stream, &st);
    if (st != cudaStreamCaptureStatusNone) return nullptr;
    size_t want = bytes + bytes / 4;
    if (want < 2 * g.ws_bytes[slot]) want = 2 * g.ws_bytes[slot];
    if (want < (size_t)(16u << 20)) want = (size_t)(16u << 20);
    void *p = nullptr;
    if (cudaMalloc(&p, want) != cudaSuccess) return nullptr;  // the current buffer stays
    ++g_lib_allocs;
    if (g.ws[slot]) g.retired.push_back(g.ws[slot]);
    g.ws[slot] = p;
    g.ws_bytes[slot] = want;
    return p;
}

// Zero-initialised arrival counters of the stream-K GEMM (self-resetting after each
// launch).  Grown like scratch(): outgrown arrays are retired, not freed.
int *counters(size_t n) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (n <= g.ctr_n) return g.ctr;
    cudaStreamCaptureStatus st = cudaStreamCaptureStatusNone;
    cudaStreamIsCapturing(g.stream, &st);
    if (st != cudaStreamCaptureStatusNone) return nullptr;
    size_t want = n < 65536 ? 65536 : n;
    if (want < 2 * g.ctr_n) want = 2 * g.ctr_n;
    int *p = nullptr;
    if (cudaMalloc(&p, want * sizeof(int)) != cudaSuccess) return nullptr;
    ++g_lib_allocs;
    if (cudaMemset(p, 0, want * sizeof(int)) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
        cudaFree(p);
        return nullptr;
    }
    if (g.ctr) g.retired.push_back(g.ctr);
    g.ctr = p;
    g.ctr_n = want;
    return p;
}

static unsigned long long g_launches = 0;
static long long g_wait_limit = -1;

long long wait_limit_override() { return g_wait_limit; }

int check_launch(const char *what) {
    ++g_launches;
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        set_error("%s: launch failed: %s", what, cudaGetErrorString(e));
        return ECPU_ERR_KERNEL;
    }
    if (sync_mode() && !capturing()) {
        e = cudaStreamSynchronize(g.stream);
        if (e != cudaSuccess) {
            set_error("%s: execution failed: %s", what, cudaGetErrorString(e));
            return ECPU_ERR_KERNEL;
        }
    }
    return ECPU_OK;
}

}  // namespace pilm

extern "C" {

// ---- device/api.h:48-53 -------------------------------------------------------------

const edevice_vtable_t *edevice_get(edevice_t dev) {
    register_defaults();
    if ((int)dev < 0 || dev >= EDEV_COUNT) return nullptr;
    return g_registry[dev].name ? &g_registry[dev] : nullptr;
}

int edevice_register(edevice_t dev, const edevice_vtable_t *vtable) {
    register_defaults();
    if ((int)dev < 0 || dev >= EDEV_COUNT || !vtable) return -1;
    g_registry[dev] = *vtable;
    return 0;
}

int edevice_set_active(edevice_t dev) {
    register_defaults();
    if ((int)dev < 0 || dev >= EDEV_COUNT || !g_registry[dev].name) return -1;
    g_active = dev;
    return 0;
}

const edevice_vtable_t *edevice_active(void) {
    register_defaults();
    return g_registry[g_active].name ? &g_registry[g_active] : nullptr;
}

int edevice_init_all(void) {
    register_defaults();
    int any = 0;
    for (int i = 0; i < EDEV_COUNT; i++) {
        if (g_registry[i].name && g_registry[i].init && !g_inited[i]) {
            if (g_registry[i].init() == 0) {
                g_inited[i] = 1;
                any = 1;
            }
        } else if (g_inited[i]) {
            any = 1;
        }
    }
    return any ? 0 : -1;
}

void edevice_shutdown_all(void) {
    for (int i = 0; i < EDEV_COUNT; i++) {
        if (g_inited[i] && g_registry[i].shutdown) g_registry[i].shutdown();
        g_inited[i] = 0;
    }
    g_active = EDEV_CUDA;
}

// ---- ecpu.h:33-39 ---------------------------------------------------------------------

ecpu_config_t ecpu_config_default(void) {
    ecpu_config_t c;
    memset(&c, 0, sizeof(c));
    c.kv_cache_budget_bytes = 4ULL * 1024 * 1024 * 1024;
    c.device_type = EDEV_CUDA;
    return c;
}

int ecpu_init(const ecpu_config_t *config) {
    if (g.initialized) {
        pilm::set_error("ecpu already initialized");
        return ECPU_ERR_PARAM;
    }
    register_defaults();
    g.config = config ? *config : ecpu_config_default();
    if (edevice_init_all() != 0) {
        pilm::set_error("device init failed");
        return ECPU_ERR_DEVICE;
    }
    if (g.config.device_type == EDEV_CUDA && !g_inited[EDEV_CUDA]) {
        pilm::set_error("no sm_100 CUDA device available");
        return ECPU_ERR_DEVICE;
    }
    if (edevice_set_active(g.config.device_type) != 0) {
        pilm::set_error("set active device failed");
        return ECPU_ERR_DEVICE;
    }
    g.initialized = 1;
    return ECPU_OK;
}

void ecpu_shutdown(void) {
    if (!g.initialized) return;
    for (int i = 0; i < pilm::kScratchSlots; i++) {
        if (g.ws[i]) cudaFree(g.ws[i]);
        g.ws[i] = nullptr;
        g.ws_bytes[i] = 0;
    }
    if (g.ctr) cudaFree(g.ctr);
    g.ctr = nullptr;
    g.ctr_n = 0;
    cudaDeviceSynchronize();
    for (void *p : g.retired) cudaFree(p);
    g.retired.clear();
    edevice_shutdown_all();
    g.initialized = 0;
    g.err[0] = 0;
}

int ecpu_is_initialized(void) { return g.initialized; }
const char *ecpu_version(void) { return PILM_VERSION_STRING; }
const char *ecpu_last_error(void) { return g.err[0] ? g.err : nullptr; }

// ---- kernel/api.h:23-24 ---------------------------------------------------------------

ekernel_isa_t ekernel_detect_isa(void) { return EKERNEL_ISA_SM100A; }

const char *ekernel_isa_name(ekernel_isa_t isa) {
    switch (isa) {
        case EKERNEL_ISA_SCALAR: return "scalar";
        case EKERNEL_ISA_AVX2: return "avx2";
        case EKERNEL_ISA_AVX512: return "avx512";
        case EKERNEL_ISA_AMX: return "amx";
        case EKERNEL_ISA_NEON: return "neon";
        case EKERNEL_ISA_SVE: return "sve";
        case EKERNEL_ISA_SM100A: return "sm_100a";
        default: return "unknown";
    }
}

// ---- stream control ---------------------------------------------------------------------

int ekernel_set_stream(void *s) {
    g.stream = (cudaStream_t)s;
    return ECPU_OK;
}

void *ekernel_get_stream(void) { return (void *)g.stream; }

unsigned long long ekernel_launch_count(void) { return pilm::g_launches; }

unsigned long long ekernel_alloc_count(void) { return pilm::g_lib_allocs; }

int ekernel_set_wait_limit(long long polls) {
    pilm::g_wait_limit = polls < 0 ? -1 : (polls > 0xffffffffll ? 0xffffffffll : polls);
    return ECPU_OK;
}

int ekernel_synchronize(void) {
    cudaError_t e = cudaStreamSynchronize(g.stream);
    if (e != cudaSuccess) {
        pilm::set_error("synchronize: %s", cudaGetErrorString(e));
        return ECPU_ERR_KERNEL;
    }
    return ECPU_OK;
}

}  // extern "C"
