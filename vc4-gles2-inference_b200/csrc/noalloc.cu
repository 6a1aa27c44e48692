// noalloc.cu -- GPU::matvec_s with no device allocation.
//
// vc4_matvec_s stages its scaled input and its integer outputs in device
// buffers it allocates and frees on every call.  Some callers cannot let a
// library do that: a host that has handed the device's memory to its own pool
// (a serving framework that owns every byte of HBM) must not see allocations
// behind its back, and a latency-critical thread cannot risk the implicit
// device synchronisation cudaMalloc/cudaFree may cause.  This variant keeps
// that scratch in one file-scope __device__ array instead.  The caller passes
// the input and output as device pointers it owns; the call allocates nothing.
//
// The array is loaded with the library on every GPU that uses it and stays
// resident until the process exits.  Its host-side name is only a stand-in:
// the device address is fetched once per device with cudaGetSymbolAddress and
// that address is what the kernels receive.
#include "vc4b200_internal.h"
#include "../../include/vc4b200.h"

#include <mutex>

namespace {

constexpr int kMaxCols = 16384;   // widest input the scratch holds
constexpr int kMaxRows = 81920;   // most output rows (the largest logits matrix here is 73448)
constexpr int kMaxDevices = 64;

struct Scratch {
    int16_t xq[kMaxCols];   // the input scaled by 2^k and quantised to q16
    int32_t v[kMaxRows];    // the clamped q16 integers of every output row
    int k;                  // the power-of-two scale exponent
};

// Every call on a device shares this one copy and it keeps the last call's
// contents.  Nothing in it has to start at zero: each call writes xq[0..cols),
// v[0..rows) and k before reading them.
static __device__ __align__(256) Scratch g_scratch;

std::mutex g_setup_mu;
Scratch* g_scratch_dev[kMaxDevices] = {};

// matvec_s input scaling (gpu_conv.cpp:271-287) on the device: k = 6 - e with
// max|x| = f*2^e, then q16(x*2^k) with lrintf's rounding.
__global__ void __launch_bounds__(256) k_scale(const float* x, int n, Scratch* sc) {
    __shared__ float red[8];
    float mx = 0.0f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) mx = fmaxf(mx, fabsf(x[i]));
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
    __syncthreads();
    mx = red[0];
    for (int w = 1; w < 8; ++w) mx = fmaxf(mx, red[w]);
    int k = 0;
    if (mx > 0.0f) {
        int e = 0;
        frexpf(mx, &e);
        k = 6 - e;
    }
    const float sk = ldexpf(1.0f, k);
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const int q = __float2int_rn(__fmul_rn(__fmul_rn(x[i], sk), 256.0f));
        sc->xq[i] = (int16_t)(q < -32768 ? -32768 : q > 32767 ? 32767 : q);
    }
    if (threadIdx.x == 0) sc->k = k;
}

// Read back: (v / 256) * 2^-k, the host arithmetic of vc4_matvec_s.
__global__ void k_unscale(const Scratch* sc, int rows, float* out) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= rows) return;
    out[r] = __fmul_rn(__fdiv_rn((float)sc->v[r], 256.0f), ldexpf(1.0f, -sc->k));
}

// The scratch address on the current device, fetched once per device.
int scratch_on(int dev, Scratch** out) {
    if (dev < 0 || dev >= kMaxDevices) return vc4::set_error(VC4_EINVAL, "matvec_s_noalloc: device index too large");
    std::lock_guard<std::mutex> lk(g_setup_mu);
    if (!g_scratch_dev[dev]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_scratch);
        if (e != cudaSuccess)
            return vc4::set_error(VC4_ECUDA, (std::string("matvec_s_noalloc: cudaGetSymbolAddress: ") +
                                              cudaGetErrorString(e)).c_str());
        g_scratch_dev[dev] = static_cast<Scratch*>(p);
    }
    *out = g_scratch_dev[dev];
    return VC4_OK;
}

}  // namespace

extern "C" int vc4_matvec_s_noalloc(vc4_model* m, int which, int layer, int expert, const float* d_x,
                                    float* d_out, void* stream) {
    int idx = -1;
    if (int e = vc4::lookup_matrix(m, which, layer, expert, &idx)) return e;
    const vc4::DModel& d = vc4::model_of(m);
    const vc4::DMat& W = d.mats[idx];
    if (W.cols > kMaxCols || W.rows > kMaxRows) {
        const std::string msg = "matvec_s_noalloc: a " + std::to_string(W.rows) + "x" + std::to_string(W.cols) +
                                " matrix exceeds the scratch limit of " + std::to_string(kMaxRows) + " rows x " +
                                std::to_string(kMaxCols) + " columns";
        return vc4::set_error(VC4_EINVAL, msg.c_str());
    }
    if (!d_x || !d_out) return vc4::set_error(VC4_EINVAL, "matvec_s_noalloc: null input or output");
    cudaError_t ce = cudaSetDevice(d.device);
    if (ce != cudaSuccess) return vc4::set_error(VC4_ECUDA, cudaGetErrorString(ce));
    Scratch* sc = nullptr;
    if (int e = scratch_on(d.device, &sc)) return e;
    cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : vc4::model_stream(m);
    k_scale<<<1, 256, 0, st>>>(d_x, W.cols, sc);
    vc4::launch_matvec_raw(d, idx, sc->xq, W.cols, sc->v, st);
    k_unscale<<<(W.rows + 255) / 256, 256, 0, st>>>(sc, W.rows, d_out);
    ce = cudaGetLastError();
    if (ce != cudaSuccess) return vc4::set_error(VC4_ECUDA, cudaGetErrorString(ce));
    return VC4_OK;
}
