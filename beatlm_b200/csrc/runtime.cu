// Error reporting, the device status word and TMA tensor-map encoding.
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "host.h"

namespace bl {

namespace {
thread_local char g_msg[1024] = "";
// One status word per device: kernels record here instead of trapping.
__device__ Status g_status;

std::mutex g_mu;
Status* g_status_addr[64] = {};

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn g_encode = nullptr;

EncodeTiledFn encode_fn() {
    std::lock_guard<std::mutex> lk(g_mu);
    if (g_encode == nullptr) {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_encode = reinterpret_cast<EncodeTiledFn>(fn);
    }
    return g_encode;
}
}  // namespace

int fail(int code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_msg, sizeof g_msg, fmt, ap);
    va_end(ap);
    return code;
}

bool pdl_enabled() {
    static const bool on = [] {
        const char* v = getenv("BEATLM_B200_PDL");
        return !(v != nullptr && v[0] == '0');
    }();
    return on;
}

Status* status_ptr() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    std::lock_guard<std::mutex> lk(g_mu);
    if (g_status_addr[dev] == nullptr) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_status) != cudaSuccess) return nullptr;
        g_status_addr[dev] = static_cast<Status*>(p);
    }
    return g_status_addr[dev];
}

static int encode(CUtensorMap* map, const void* base, cuuint32_t rank, const cuuint64_t* dims,
                  const cuuint64_t* strides, const cuuint32_t* box,
                  CUtensorMapDataType dtype = CU_TENSOR_MAP_DATA_TYPE_UINT16,
                  CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
    EncodeTiledFn fn = encode_fn();
    if (fn == nullptr) return fail(BL_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
    if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0)
        return fail(BL_ERR_INVALID, "tensor base %p is not 16-byte aligned", base);
    for (cuuint32_t i = 0; i + 1 < rank; ++i)
        if (strides[i] % 16 != 0)
            return fail(BL_ERR_INVALID, "tensor stride %llu is not a multiple of 16 bytes",
                        (unsigned long long)strides[i]);
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = fn(map, dtype, rank, const_cast<void*>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(BL_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return BL_OK;
}

int make_tmap_16bit_3d(CUtensorMap* map, const void* base, const uint64_t dims[3],
                       const uint64_t strides_bytes[2], const uint32_t box[3]) {
    cuuint64_t d[3] = {dims[0], dims[1], dims[2]};
    cuuint64_t s[2] = {strides_bytes[0], strides_bytes[1]};
    cuuint32_t b[3] = {box[0], box[1], box[2]};
    return encode(map, base, 3, d, s, b);
}

int make_tmap_2d(CUtensorMap* map, const void* base, int esz, const uint64_t dims[2],
                 uint64_t row_stride_bytes, const uint32_t box[2], int swizzle_bytes) {
    cuuint64_t d[2] = {dims[0], dims[1]};
    cuuint64_t s[1] = {row_stride_bytes};
    cuuint32_t b[2] = {box[0], box[1]};
    return encode(map, base, 2, d, s, b,
                  esz == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_UINT16,
                  swizzle_bytes == 128  ? CU_TENSOR_MAP_SWIZZLE_128B
                  : swizzle_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                        : CU_TENSOR_MAP_SWIZZLE_NONE);
}

int make_tmap_16bit_2d(CUtensorMap* map, const void* base, const uint64_t dims[2],
                       uint64_t row_stride_bytes, const uint32_t box[2]) {
    cuuint64_t d[2] = {dims[0], dims[1]};
    cuuint64_t s[1] = {row_stride_bytes};
    cuuint32_t b[2] = {box[0], box[1]};
    return encode(map, base, 2, d, s, b);
}

}  // namespace bl

extern "C" size_t bl_last_error(char* buf, size_t cap) {
    size_t n = strlen(bl::g_msg);
    if (buf != nullptr && cap > 0) {
        size_t c = n < cap - 1 ? n : cap - 1;
        memcpy(buf, bl::g_msg, c);
        buf[c] = '\0';
    }
    return n;
}

extern "C" const char* bl_version(void) { return "beatlm-b200 0.1 sm_100a"; }

extern "C" int bl_status(bl_status_t* out, int reset) {
    bl::Status* p = bl::status_ptr();
    if (p == nullptr) return bl::fail(BL_ERR_CUDA, "no device status word on this device");
    BL_CUDA_TRY(cudaDeviceSynchronize());
    bl::Status s{};
    BL_CUDA_TRY(cudaMemcpy(&s, p, bl::kStatusReportBytes, cudaMemcpyDeviceToHost));
    if (out != nullptr) {
        out->code = s.code;
        out->block = s.block;
        out->where = s.where;
        out->count = s.count;
    }
    // the error fields only: the wait limit stays as the host set it
    if (reset) BL_CUDA_TRY(cudaMemset(p, 0, bl::kStatusReportBytes));
    return BL_OK;
}

extern "C" int bl_set_wait_limit(uint64_t cycles) {
    bl::Status* p = bl::status_ptr();
    if (p == nullptr) return bl::fail(BL_ERR_CUDA, "no device status word on this device");
    if (cycles > 60ull * 1965ull * 1000ull * 1000ull)
        return bl::fail(BL_ERR_INVALID, "wait limit %llu cycles (at most about 60 s)",
                        (unsigned long long)cycles);
    unsigned long long v = cycles;
    // ordered after earlier work on the legacy stream and before later launches
    BL_CUDA_TRY(cudaMemcpy(&p->limit_cycles, &v, sizeof v, cudaMemcpyHostToDevice));
    return BL_OK;
}

extern "C" uint64_t bl_wait_limit(void) {
    bl::Status* p = bl::status_ptr();
    unsigned long long v = 0;
    if (p == nullptr || cudaMemcpy(&v, &p->limit_cycles, sizeof v, cudaMemcpyDeviceToHost) !=
                            cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return v;
}

namespace bl {
// One warp that waits `ns` nanoseconds of %globaltimer time and exits. The
// loop ends by construction (the wait is bounded by the argument, at most
// one second, checked on the host).
__global__ void hold_kernel(uint64_t ns) {
    uint64_t t0, t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
    do {
        __nanosleep(2000);
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    } while (t - t0 < ns);
}
}  // namespace bl

extern "C" int bl_stream_hold(void* stream, uint32_t microseconds) {
    if (microseconds > 1000000)
        return bl::fail(BL_ERR_INVALID, "stream hold: %u us (max 1 s)", microseconds);
    bl::hold_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(1000ull * microseconds);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return bl::fail(BL_ERR_CUDA, "stream hold: %s", cudaGetErrorString(e));
    return BL_OK;
}
