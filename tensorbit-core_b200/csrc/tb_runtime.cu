// Library runtime: error reporting, device plumbing and the per-device caches
// (top-N tie tables, host-path staging buffers).
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <tuple>
#include <vector>

#include "tb_runtime.h"

namespace tb {

std::vector<uint8_t> build_topn_table(int n, int m);  // tb_lut.cpp

namespace {
thread_local std::string t_last_error;

struct TableKey {
    int dev, n, m;
    bool operator<(const TableKey& o) const { return std::tie(dev, n, m) < std::tie(o.dev, o.n, o.m); }
};

std::mutex g_mu;
std::map<TableKey, uint8_t*> g_tables;
}  // namespace

namespace {
std::mutex g_pool_mu;
std::map<int, cudaMemPool_t> g_pools;
}  // namespace

int scratch_alloc(void** ptr, size_t bytes, cudaStream_t stream) {
    int dev = 0;
    int rc = require_device(&dev);
    if (rc) return rc;
    cudaMemPool_t pool = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_pool_mu);
        auto it = g_pools.find(dev);
        if (it == g_pools.end()) {
            cudaMemPoolProps props{};
            props.allocType = cudaMemAllocationTypePinned;
            props.location.type = cudaMemLocationTypeDevice;
            props.location.id = dev;
            cudaError_t e = cudaMemPoolCreate(&pool, &props);
            if (e != cudaSuccess) return cuda_fail(e, "cudaMemPoolCreate(scratch)");
            uint64_t keep = UINT64_MAX;
            e = cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep);
            if (e != cudaSuccess) return cuda_fail(e, "cudaMemPoolSetAttribute(scratch)");
            g_pools[dev] = pool;
        } else {
            pool = it->second;
        }
    }
    cudaError_t e = cudaMallocFromPoolAsync(ptr, bytes, pool, stream);
    return e == cudaSuccess ? TB_OK : cuda_fail(e, "cudaMallocFromPoolAsync(scratch)");
}

void scratch_free(void* ptr, cudaStream_t stream) {
    if (ptr) cudaFreeAsync(ptr, stream);
}

int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    std::vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    t_last_error = buf;
    return code;
}

int cuda_fail(cudaError_t e, const char* what) {
    return fail(TB_ERR_CUDA, "%s: %s (%d)", what, cudaGetErrorString(e), static_cast<int>(e));
}

int check_launch(const char* what) {
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? TB_OK : cuda_fail(e, what);
}

int require_device(int* dev_out) {
    int count = 0;
    cudaError_t e = cudaGetDeviceCount(&count);
    if (e != cudaSuccess || count == 0) {
        cudaGetLastError();
        return fail(TB_ERR_NO_DEVICE, "no CUDA device available (%s)", cudaGetErrorString(e));
    }
    int dev = 0;
    e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    if (dev_out) *dev_out = dev;
    return TB_OK;
}

int topn_table(int n, int m, const uint8_t** out) {
    int dev = 0;
    int rc = require_device(&dev);
    if (rc) return rc;
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_tables.find({dev, n, m});
    if (it != g_tables.end()) { *out = it->second; return TB_OK; }
    std::vector<uint8_t> host = build_topn_table(n, m);
    uint8_t* d = nullptr;
    cudaError_t e = cudaMalloc(&d, host.size());
    if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(top-N tie table)");
    e = cudaMemcpy(d, host.data(), host.size(), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) { cudaFree(d); return cuda_fail(e, "cudaMemcpy(top-N tie table)"); }
    g_tables[{dev, n, m}] = d;
    *out = d;
    return TB_OK;
}

bool topn_table_ready(int n, int m) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return false;
    std::lock_guard<std::mutex> lk(g_mu);
    return g_tables.count({dev, n, m}) != 0;
}

}  // namespace tb

using namespace tb;

extern "C" {

int tb_abi_version(void) { return TB_ABI_VERSION; }

const char* tb_last_error(void) { return t_last_error.c_str(); }

int tb_device_count(int* count) {
    if (!count) return fail(TB_ERR_ARG, "tb_device_count: null pointer");
    int c = 0;
    cudaError_t e = cudaGetDeviceCount(&c);
    if (e != cudaSuccess) { cudaGetLastError(); c = 0; }
    *count = c;
    return TB_OK;
}

int tb_set_device(int device) {
    int rc = require_device(nullptr);
    if (rc) return rc;
    cudaError_t e = cudaSetDevice(device);
    return e == cudaSuccess ? TB_OK : cuda_fail(e, "cudaSetDevice");
}

int tb_malloc(void** ptr, size_t bytes) {
    if (!ptr) return fail(TB_ERR_ARG, "tb_malloc: null pointer");
    *ptr = nullptr;
    int rc = require_device(nullptr);
    if (rc) return rc;
    if (bytes == 0) return TB_OK;
    cudaError_t e = cudaMalloc(ptr, bytes);
    return e == cudaSuccess ? TB_OK : cuda_fail(e, "cudaMalloc");
}

int tb_host_alloc(void** ptr, size_t bytes) {
    if (!ptr) return fail(TB_ERR_ARG, "tb_host_alloc: null pointer");
    *ptr = nullptr;
    int rc = require_device(nullptr);
    if (rc) return rc;
    if (bytes == 0) return TB_OK;
    cudaError_t e = cudaHostAlloc(ptr, bytes, cudaHostAllocPortable);
    return e == cudaSuccess ? TB_OK : cuda_fail(e, "cudaHostAlloc");
}

int tb_host_free(void* ptr) {
    if (!ptr) return TB_OK;
    cudaError_t e = cudaFreeHost(ptr);
    return e == cudaSuccess ? TB_OK : cuda_fail(e, "cudaFreeHost");
}

int tb_free(void* ptr) {
    if (!ptr) return TB_OK;
    cudaError_t e = cudaFree(ptr);
    return e == cudaSuccess ? TB_OK : cuda_fail(e, "cudaFree");
}

static int copy(void* dst, const void* src, size_t bytes, cudaMemcpyKind kind, void* stream, const char* what) {
    if (bytes == 0) return TB_OK;
    if (!dst || !src) return fail(TB_ERR_ARG, "%s: null pointer", what);
    int rc = require_device(nullptr);
    if (rc) return rc;
    cudaError_t e = cudaMemcpyAsync(dst, src, bytes, kind, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? TB_OK : cuda_fail(e, what);
}

int tb_memcpy_h2d(void* dst, const void* src, size_t bytes, void* stream) {
    return copy(dst, src, bytes, cudaMemcpyHostToDevice, stream, "tb_memcpy_h2d");
}
int tb_memcpy_d2h(void* dst, const void* src, size_t bytes, void* stream) {
    return copy(dst, src, bytes, cudaMemcpyDeviceToHost, stream, "tb_memcpy_d2h");
}
int tb_memcpy_d2d(void* dst, const void* src, size_t bytes, void* stream) {
    return copy(dst, src, bytes, cudaMemcpyDeviceToDevice, stream, "tb_memcpy_d2d");
}

int tb_memset(void* dst, int value, size_t bytes, void* stream) {
    if (bytes == 0) return TB_OK;
    if (!dst) return fail(TB_ERR_ARG, "tb_memset: null pointer");
    int rc = require_device(nullptr);
    if (rc) return rc;
    cudaError_t e = cudaMemsetAsync(dst, value, bytes, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? TB_OK : cuda_fail(e, "tb_memset");
}

int tb_stream_sync(void* stream) {
    int rc = require_device(nullptr);
    if (rc) return rc;
    cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? TB_OK : cuda_fail(e, "cudaStreamSynchronize");
}

int tb_ipc_handle(const void* dev_ptr, void* handle_out) {
    if (!dev_ptr || !handle_out) return fail(TB_ERR_ARG, "tb_ipc_handle: null pointer");
    int rc = require_device(nullptr);
    if (rc) return rc;
    static_assert(sizeof(cudaIpcMemHandle_t) == TB_IPC_HANDLE_BYTES, "IPC handle size");
    cudaIpcMemHandle_t h;
    cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void*>(dev_ptr));
    if (e != cudaSuccess) return cuda_fail(e, "cudaIpcGetMemHandle");
    std::memcpy(handle_out, &h, sizeof(h));
    return TB_OK;
}

int tb_ipc_open(const void* handle, void** dev_ptr_out) {
    if (!handle || !dev_ptr_out) return fail(TB_ERR_ARG, "tb_ipc_open: null pointer");
    *dev_ptr_out = nullptr;
    int rc = require_device(nullptr);
    if (rc) return rc;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    cudaError_t e = cudaIpcOpenMemHandle(dev_ptr_out, h, cudaIpcMemLazyEnablePeerAccess);
    return e == cudaSuccess ? TB_OK : cuda_fail(e, "cudaIpcOpenMemHandle");
}

int tb_ipc_close(void* dev_ptr) {
    if (!dev_ptr) return TB_OK;
    cudaError_t e = cudaIpcCloseMemHandle(dev_ptr);
    return e == cudaSuccess ? TB_OK : cuda_fail(e, "cudaIpcCloseMemHandle");
}

int tb_enable_peer_access(int peer_device) {
    int rc = require_device(nullptr);
    if (rc) return rc;
    int dev = 0, can = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceCanAccessPeer(&can, dev, peer_device);
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceCanAccessPeer");
    if (peer_device == dev) return TB_OK;
    if (!can) return fail(TB_ERR_UNSUPPORTED, "device %d cannot access device %d", dev, peer_device);
    e = cudaDeviceEnablePeerAccess(peer_device, 0);
    if (e == cudaErrorPeerAccessAlreadyEnabled) {
        cudaGetLastError();
        return TB_OK;
    }
    return e == cudaSuccess ? TB_OK : cuda_fail(e, "cudaDeviceEnablePeerAccess");
}

int tb_prepare_nm(int n, int m) {
    if (n <= 0 || m <= 0 || n >= m) return fail(TB_ERR_CONFIG, "invalid N:M %d:%d", n, m);
    if (m > 8) return fail(TB_ERR_UNSUPPORTED, "M=%d > 8: masks hold one byte per group", m);
    const uint8_t* t = nullptr;
    return topn_table(n, m, &t);
}

}  // extern "C"
