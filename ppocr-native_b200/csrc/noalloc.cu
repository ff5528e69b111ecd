// ppocr_ctc_argmax_noalloc: the CTC argmax head for callers that may not
// allocate device memory.
//
// Some hosts own every byte of device memory themselves (an inference server
// with a fixed memory budget, a plugin host that forbids allocation from
// plugin code) or run loops that must never stall, and cudaMalloc / cudaFree
// can synchronize the whole device. Such callers cannot use the model API,
// which allocates its tensors and scratch in ppocr_model_set_sizes. This entry
// point runs the same CTC argmax kernels as the model path over buffers the
// caller passes in, and keeps the one scratch buffer those kernels need — the
// per-pixel, per-column-block (max, sum, best column) states — in a
// fixed-size array in the library's own device memory.
//
// That array is a file-scope __device__ variable: every GPU that loads the
// library holds its NOALLOC_SCRATCH_FLOATS floats (4 MiB) until the process
// exits, and every call on a device uses the same array, so calls that
// overlap on the GPU (on different streams, or from several threads without
// ordering) race on it. Nothing in it has to start at zero: the logits kernel
// writes every state the merge kernel then reads. The array keeps the last
// call's contents.
//
// Host code cannot pass the array's name to a kernel (on the host that name
// is only a stand-in for the device variable); its device address comes from
// cudaGetSymbolAddress, once per device, with that device current. The same
// once-per-device set-up raises the logits kernel's dynamic shared-memory
// limit on that device (the head's ci x (64 + 128) floats of staging exceed
// the 48 KB default for ci > 64), so a process that never builds a model can
// call this entry point. The first call on each device does that set-up, so
// that first call should come before any stream capture. No call allocates:
// no cudaMalloc, cudaFree or allocating library routine is used here.
//
// The logits kernel reads the weight panels as 16-byte vectors, so `w` must
// be 16-byte aligned; the other buffers are read and written as floats. A
// misaligned pointer is refused before any launch (PPOCR_E_ARG) rather than
// faulting on the device.
#include <cuda_runtime.h>

#include <cstdint>
#include <map>
#include <mutex>
#include <string>

#include "../../include/ppocr_cuda.h"
#include "kernels.hpp"

namespace ppocr {
void set_last_error(const std::string &msg);
}

using namespace ppocr;

namespace {

// 1 Mi floats: three floats per (time step, 128-column block), enough for
// 2377 time steps of the 18 710-class head (about 23 lines of 48 x 820) per call.
constexpr size_t NOALLOC_SCRATCH_FLOATS = size_t(1) << 20;

static __device__ __align__(256) float g_ctc_scratch[NOALLOC_SCRATCH_FLOATS];

// The array's device address on the current device, looked up once, and
// the kernels' limits raised on that device at the same time.
int scratch_on_device(float **out) {
    static std::mutex mu;
    static std::map<int, float *> by_device;
    int device = 0;
    cudaError_t e = cudaGetDevice(&device);
    if (e != cudaSuccess) {
        set_last_error(std::string("ppocr_ctc_argmax_noalloc: no current device: ") + cudaGetErrorString(e));
        return PPOCR_E_DEVICE;
    }
    std::lock_guard<std::mutex> lock(mu);
    auto it = by_device.find(device);
    if (it != by_device.end()) {
        *out = it->second;
        return PPOCR_OK;
    }
    float *ptr = nullptr;
    e = cudaGetSymbolAddress(reinterpret_cast<void **>(&ptr), g_ctc_scratch);
    if (e != cudaSuccess || !ptr) {
        set_last_error(std::string("ppocr_ctc_argmax_noalloc: locating the scratch array: ") +
                       cudaGetErrorString(e));
        return PPOCR_E_DEVICE;
    }
    configure_misc_kernels();
    e = cudaGetLastError();
    if (e != cudaSuccess) {
        set_last_error(std::string("ppocr_ctc_argmax_noalloc: raising the kernels' shared-memory limits: ") +
                       cudaGetErrorString(e));
        return PPOCR_E_DEVICE;
    }
    by_device[device] = ptr;
    *out = ptr;
    return PPOCR_OK;
}

}  // namespace

extern "C" int ppocr_ctc_argmax_noalloc(const float *x, const float *w, const float *b, float *y, size_t pixels,
                                        size_t ci, size_t vocab, void *stream) {
    set_last_error("");
    if (!x || !w || !b || !y || pixels == 0 || ci == 0 || vocab == 0) {
        set_last_error("ppocr_ctc_argmax_noalloc: null buffer or empty size");
        return PPOCR_E_ARG;
    }
    const auto misaligned = [](const void *p, uintptr_t n) { return (reinterpret_cast<uintptr_t>(p) & (n - 1)) != 0; };
    if (misaligned(w, 16) || misaligned(x, 4) || misaligned(b, 4) || misaligned(y, 4)) {
        set_last_error("ppocr_ctc_argmax_noalloc: w must be 16-byte aligned and x, b, y 4-byte aligned");
        return PPOCR_E_ARG;
    }
    size_t cols = (vocab + 15) / 16 * 16;
    size_t blocks = size_t(ctc_col_blocks(int(cols)));
    if (!ctc_supported(int(ci > (size_t(1) << 20) ? (size_t(1) << 20) : ci))) {
        set_last_error("ppocr_ctc_argmax_noalloc: " + std::to_string(ci) + " input channels exceed this backend");
        return PPOCR_E_SIZE;
    }
    if (pixels > size_t(1) << 30 || ci > (size_t(1) << 20) || vocab > (size_t(1) << 24) ||
        pixels * blocks * 3 > NOALLOC_SCRATCH_FLOATS) {
        set_last_error("ppocr_ctc_argmax_noalloc: " + std::to_string(pixels) + " time steps x " +
                       std::to_string(vocab) + " classes need " + std::to_string(pixels * blocks * 3) +
                       " scratch floats, more than the " + std::to_string(NOALLOC_SCRATCH_FLOATS) +
                       " this entry point holds; split the call");
        return PPOCR_E_SIZE;
    }
    float *scratch = nullptr;
    int rc = scratch_on_device(&scratch);
    if (rc) return rc;
    CtcArgs a;
    a.x = x;
    a.w = w;
    a.b = b;
    a.y = y;
    a.partial = scratch;
    a.pixels = int(pixels);
    a.ci = int(ci);
    a.vocab = int(vocab);
    a.cols = int(cols);
    a.col_blocks = int(blocks);
    a.probs = false;
    launch_ctc(a, static_cast<cudaStream_t>(stream));
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        set_last_error(std::string("ppocr_ctc_argmax_noalloc: launching: ") + cudaGetErrorString(e));
        return PPOCR_E_DEVICE;
    }
    return PPOCR_OK;
}
