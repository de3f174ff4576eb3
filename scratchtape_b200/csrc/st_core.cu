// st_core.cu -- handle lifecycle, error text, scratch pool, tensor maps.
#include <cstring>
#include <mutex>

#include "st_internal.h"
#include "st_ptx.cuh"

extern "C" st_status st_create(int device, void *stream, st_handle **out) {
    if (!out) return ST_INVALID_ARG;
    *out = nullptr;
    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess || device < 0 || device >= count) return ST_INVALID_ARG;
    if (cudaSetDevice(device) != cudaSuccess) return ST_CUDA_ERROR;
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) return ST_CUDA_ERROR;
    if (prop.major != 10) return ST_UNSUPPORTED_SHAPE;  // sm_100a only
    st_handle *h = new st_handle();
    h->device = device;
    h->stream = static_cast<cudaStream_t>(stream);
    h->num_sms = prop.multiProcessorCount;
    if (cudaMalloc(&h->d_status, sizeof(int)) != cudaSuccess) {
        delete h;
        return ST_NO_MEMORY;
    }
    if (cudaMemset(h->d_status, 0, sizeof(int)) != cudaSuccess) {
        cudaFree(h->d_status);
        delete h;
        return ST_CUDA_ERROR;
    }
    *out = h;
    return ST_OK;
}

extern "C" st_status st_destroy(st_handle *h) {
    if (!h) return ST_INVALID_ARG;
    cudaSetDevice(h->device);
    cudaStreamSynchronize(h->stream);
    for (int i = 0; i < SLOT_COUNT; i++)
        if (h->slot_ptr[i]) cudaFree(h->slot_ptr[i]);
    if (h->d_status) cudaFree(h->d_status);
    delete h;
    return ST_OK;
}

extern "C" st_status st_set_stream(st_handle *h, void *stream) {
    if (!h) return ST_INVALID_ARG;
    h->stream = static_cast<cudaStream_t>(stream);
    return ST_OK;
}

extern "C" const char *st_last_error(const st_handle *h) { return h ? h->err.c_str() : "null handle"; }

extern "C" int64_t st_launch_count(const st_handle *h) { return h ? h->launches : 0; }

extern "C" const char *st_last_kernel(const st_handle *h) { return h ? h->last_kernel : ""; }

extern "C" int64_t st_scratch_bytes(const st_handle *h) {
    if (!h) return 0;
    int64_t s = 0;
    for (int i = 0; i < SLOT_COUNT; i++) s += static_cast<int64_t>(h->slot_bytes[i]);
    return s;
}

extern "C" st_status st_sync(st_handle *h) {
    if (!h) return ST_INVALID_ARG;
    ST_CHECK_CUDA(h, cudaStreamSynchronize(h->stream));
    int status = 0;
    ST_CHECK_CUDA(h, cudaMemcpy(&status, h->d_status, sizeof(int), cudaMemcpyDeviceToHost));
    if (status != 0) {
        ST_CHECK_CUDA(h, cudaMemset(h->d_status, 0, sizeof(int)));
        if (status == st::DEV_BAD_ARG) return h->fail(ST_INVALID_ARG, "a kernel met an out-of-range index");
        return h->fail(ST_TIMEOUT, "device-side bounded wait ran out (code %d)", status);
    }
    return ST_OK;
}

st_status st_after_launch(st_handle *h, const char *what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return h->fail(ST_CUDA_ERROR, "launch of %s failed: %s", what, cudaGetErrorString(e));
    h->launches++;
    h->last_kernel = what;
    return ST_OK;
}

void *st_scratch(st_handle *h, int slot, size_t bytes) {
    if (slot < 0 || slot >= SLOT_COUNT) return nullptr;
    if (bytes == 0) bytes = 256;
    if (h->slot_bytes[slot] >= bytes) return h->slot_ptr[slot];
    if (h->slot_ptr[slot]) {
        // the stream may still read the old buffer
        if (cudaStreamSynchronize(h->stream) != cudaSuccess) {
            h->fail(ST_CUDA_ERROR, "scratch growth: stream sync failed");
            return nullptr;
        }
        cudaFree(h->slot_ptr[slot]);
        h->slot_ptr[slot] = nullptr;
        h->slot_bytes[slot] = 0;
    }
    size_t want = bytes + bytes / 8;
    want = (want + 4095) / 4096 * 4096;
    void *p = nullptr;
    if (cudaMalloc(&p, want) != cudaSuccess) {
        cudaGetLastError();
        h->fail(ST_NO_MEMORY, "scratch slot %d: cudaMalloc(%zu) failed", slot, want);
        return nullptr;
    }
    h->slot_ptr[slot] = p;
    h->slot_bytes[slot] = want;
    return p;
}

PFN_cuTensorMapEncodeTiled_v12000 st_encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

bool st_make_map_4d(CUtensorMap *map, CUtensorMapDataType dtype, int elem_bytes, const void *base, uint64_t cols,
                    uint64_t rows, uint64_t grp, uint64_t outer, uint64_t ld_elems, uint64_t inner_elems,
                    uint64_t stride_elems, uint32_t box_cols, uint32_t box_rows, CUtensorMapSwizzle swz,
                    std::string *why) {
    auto enc = st_encode_fn();
    if (!enc) {
        if (why) *why = "cuTensorMapEncodeTiled unavailable";
        return false;
    }
    if (reinterpret_cast<uintptr_t>(base) % 16 != 0) {
        if (why) *why = "matrix start not 16-byte aligned";
        return false;
    }
    cuuint64_t dims[4] = {cols, rows, grp, outer};
    cuuint64_t strides[3] = {ld_elems * elem_bytes, inner_elems * elem_bytes, stride_elems * elem_bytes};
    for (int i = 0; i < 3; i++) {
        if (strides[i] % 16 != 0 || strides[i] == 0 || strides[i] >= (1ull << 40)) {
            if (why) *why = "tensor stride not a nonzero multiple of 16 bytes";
            return false;
        }
    }
    cuuint32_t box[4] = {box_cols, box_rows, 1, 1};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    CUresult r = enc(map, dtype, 4, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        if (why) *why = "cuTensorMapEncodeTiled rejected the layout";
        return false;
    }
    return true;
}
