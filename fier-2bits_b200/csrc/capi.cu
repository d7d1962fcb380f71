// Error reporting, version and small utility entry points of the C ABI.
#include <cstring>

#include "common.cuh"

namespace popkv {

static thread_local char g_last_error[512] = "";

void set_error(const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_last_error, sizeof g_last_error, fmt, ap);
    va_end(ap);
}

int fail(int status, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_last_error, sizeof g_last_error, fmt, ap);
    va_end(ap);
    return status;
}

int check_launch(const char* what) {
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(POPKV_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
    return POPKV_OK;
}

namespace {
__global__ void advance_kernel(int32_t* seq_len, int64_t batch, int32_t inc) {
    pdl_trigger();
    pdl_wait();
    const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (i < batch) seq_len[i] += inc;
}
}  // namespace

}  // namespace popkv

using namespace popkv;

extern "C" const char* popkv_error_string(int status) {
    switch (status) {
        case POPKV_OK: return "success";
        case POPKV_ERR_INVALID_ARGUMENT: return "invalid argument";
        case POPKV_ERR_CAPACITY: return "capacity exceeded";
        case POPKV_ERR_UNSUPPORTED: return "unsupported shape or dtype";
        case POPKV_ERR_ALIGNMENT: return "misaligned pointer";
        case POPKV_ERR_CUDA: return "CUDA error";
        case POPKV_ERR_WORKSPACE: return "workspace too small";
        default: return "unknown status";
    }
}

extern "C" const char* popkv_last_error(void) { return g_last_error; }

extern "C" int popkv_version(void) { return 100; }

extern "C" int popkv_advance(int32_t* seq_len, int64_t batch, int32_t increment,
                             popkv_stream_t stream) {
    if (batch < 0 || (batch > 0 && seq_len == nullptr))
        return fail(POPKV_ERR_INVALID_ARGUMENT, "seq_len must hold batch entries");
    if (batch == 0) return POPKV_OK;
    launch_pdl(advance_kernel, dim3((unsigned)((batch + 255) / 256)), dim3(256), 0, as_stream(stream),
               seq_len, batch, increment);
    return check_launch("popkv_advance");
}
