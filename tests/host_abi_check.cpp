// A C++ host of the public C ABI, built and run by tests/test_host_abi_cpu.py on a machine without a
// GPU: every header compiles in one C++ translation unit, the program links against
// libiq4xs_b200.so, and the calls below return before any CUDA work (the ggml hook's can_handle
// gates, status strings, workspace sizing, argument validation).  Prints "ok" or the first failure.
#include <cstdio>
#include <cstring>

#include "iq4xs.h"
#include "iq4xs_bench.h"
#include "iq4xs_decoder.h"
#include "iq4xs_peer.h"

#define CHECK(cond)                                                 \
    do {                                                            \
        if (!(cond)) {                                              \
            std::printf("FAILED line %d: %s\n", __LINE__, #cond);  \
            return 1;                                               \
        }                                                           \
    } while (0)

int main() {
    CHECK(iq4xs_version() == 100);
    // the ggml MUL_MAT hook's gates (patches/0001-gfx1100-mul-mat-custom.patch:148-151, 274-277)
    CHECK(custom_gemv_iq4xs_can_handle(5120, 17408, 1, IQ4XS_GGML_TYPE_IQ4_XS));
    CHECK(custom_gemv_iq4xs_can_handle(17408, 5120, IQ4XS_MAX_GEMV_BATCH, IQ4XS_GGML_TYPE_IQ4_XS));
    CHECK(!custom_gemv_iq4xs_can_handle(5120, 17408, IQ4XS_MAX_GEMV_BATCH + 1, IQ4XS_GGML_TYPE_IQ4_XS));
    CHECK(!custom_gemv_iq4xs_can_handle(4000, 4096, 1, IQ4XS_GGML_TYPE_IQ4_XS));
    CHECK(!custom_gemv_iq4xs_can_handle(4096, 4096, 1, 12));
    CHECK(custom_gemm_iq4xs_can_handle(5120, 17408, 2048, IQ4XS_GGML_TYPE_IQ4_XS));
    CHECK(!custom_gemm_iq4xs_can_handle(5120, 17408, 8, IQ4XS_GGML_TYPE_IQ4_XS));
    // a dispatch the hook would refuse comes back as an error the caller falls back on
    float x = 0.f, y = 0.f;
    CHECK(custom_gemv_iq4xs_dispatch(reinterpret_cast<void*>(0x10000), &x, &y, 4000, 16, nullptr) != cudaSuccess);
    CHECK(custom_gemv_iq4xs_dispatch(nullptr, &x, &y, 4096, 16, nullptr) != cudaSuccess);
    // status codes and their strings
    CHECK(std::strcmp(iq4xs_status_string(IQ4XS_OK), "ok") == 0);
    CHECK(std::strcmp(iq4xs_status_string(IQ4XS_ERR_WORKSPACE_TOO_SMALL), "workspace too small") == 0);
    // workspace sizing and validation of the workspace entry points
    const size_t need = iq4xs_gemv_workspace_bytes(5120, 8192, 2);
    CHECK(need >= iq4xs_q8_1_bytes(5120, 2));
    void* fake = reinterpret_cast<void*>(0x10000);
    CHECK(iq4xs_gemv_f32(nullptr, static_cast<const float*>(fake), static_cast<float*>(fake), 5120, 8192, 2, fake,
                         need, nullptr) == IQ4XS_ERR_INVALID_ARGUMENT);
    CHECK(iq4xs_gemv_f32(fake, static_cast<const float*>(fake), static_cast<float*>(fake), 5120, 8192, 2, fake,
                         need - 1, nullptr) == IQ4XS_ERR_WORKSPACE_TOO_SMALL);
    CHECK(iq4xs_gemv_f32(fake, static_cast<const float*>(fake), static_cast<float*>(fake), 5120, 8192, 9, fake,
                         need, nullptr) == IQ4XS_ERR_UNSUPPORTED_SHAPE);
    CHECK(iq4xs_q8_1_bytes(5120, 3) == 3u * 160u * 36u);
    std::printf("ok\n");
    return 0;
}
