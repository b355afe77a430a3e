// tb_matmul_i8_noalloc: the int8 MATMUL (+ fused RESCALE) for callers that
// cannot allocate device memory.
//
// Some hosts of this library may not call cudaMalloc at all: code running in
// a process whose device memory is owned by another allocator (a framework's
// caching pool that must see every allocation), code inside a region that
// forbids allocation (for example while another component holds the device's
// memory budget), or embedders that only hand over pre-sized input and output
// buffers. The regular MATMUL entry points allocate per-plan device scratch
// (the B column terms used for the a zero point, the packed RESCALE constants
// and the error word); this entry point keeps all of that in
// one file-scope device array instead, so it performs no allocation. The
// caller still passes inputs and outputs.
//
// The array is a fixed 2 MiB per device that loads this library (every GPU
// holds it until the process exits), which bounds the shapes: n*w <= 131072
// when a_zp != 0 and at most 16384 rescale channels. Shapes whose B rows are
// not 16-byte multiples (w % 16 != 0) and unaligned operands run the direct
// kernel, which needs no scratch beyond the error word: the tensor-core path
// for such B copies it into padded rows, a buffer this entry point does not
// have. The array's device address is resolved once per device and kept, so
// the entry point assumes the device's primary context is not reset
// (cudaDeviceReset) while the process uses it. Every call shares it and
// it keeps the last call's contents: each call clears the error word first. Calls that overlap on the GPU (other streams, other host
// threads) race on the array; serialise them.
#include <cuda_runtime.h>

#include <cstring>
#include <mutex>
#include <vector>

#include "internal.hpp"
#include "quant.cuh"

namespace {

constexpr size_t kScratchBytes = 2u << 20;
constexpr size_t kColtermOffset = 256;                 // after the error word (0)
constexpr long long kMaxColterm = 131072;              // n * w when a_zp != 0
constexpr int kMaxRescaleChannels = 16384;             // per-channel RESCALE multipliers / shifts
constexpr size_t kBlobOffset = kColtermOffset + sizeof(int32_t) * (kMaxColterm + 256);
constexpr size_t kMaxBlobWords = (kScratchBytes - kBlobOffset) / sizeof(int32_t);
constexpr int kMaxDevices = 64;

// Device-side scratch. In host code `g_noalloc_scratch` only names a host-side
// stand-in: its device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

struct DeviceSetup {
    bool ready = false;
    unsigned char* scratch = nullptr;
    int num_sms = 0;
    long long timeout_cycles = 0;
};
DeviceSetup g_setup[kMaxDevices];
std::mutex g_setup_mu;

// Once per device, with that device current: resolve the array's device address.
tb_status device_setup(int dev, DeviceSetup* out) {
    std::lock_guard<std::mutex> lock(g_setup_mu);
    DeviceSetup& s = g_setup[dev];
    if (!s.ready) {
        void* ptr = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
        if (e != cudaSuccess)
            return tb::fail(TB_ERR_CUDA, "cudaGetSymbolAddress(no-alloc scratch) failed: %s", cudaGetErrorString(e));
        int sms = 0, clock_khz = 0;
        e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (e == cudaSuccess) e = cudaDeviceGetAttribute(&clock_khz, cudaDevAttrClockRate, dev);
        if (e != cudaSuccess) return tb::fail(TB_ERR_CUDA, "device query failed: %s", cudaGetErrorString(e));
        s.scratch = static_cast<unsigned char*>(ptr);
        s.num_sms = sms;
        s.timeout_cycles = static_cast<long long>(2.0 * clock_khz * 1e3);  // about 2 s of bounded waiting
        s.ready = true;
    }
    *out = s;
    return TB_OK;
}

}  // namespace

extern "C" TB_API tb_status tb_matmul_i8_noalloc(const tb_matmul_desc* d, const tb_rescale_attr* rescale,
                                                 const void* a, const void* b, void* out, void* stream_) {
    using namespace tb;
    if (!d || !a || !b || !out) return fail(TB_ERR_INVALID_ARGUMENT, "null argument");
    if (d->a_dtype != TB_DT_INT8 || d->b_dtype != TB_DT_INT8 || d->out_dtype != TB_DT_INT32)
        return fail(TB_ERR_NOT_ACCELERATED, "tb_matmul_i8_noalloc runs INT8 x INT8 -> INT32 only");
    int path = 0, bn = 256;
    TB_TRY(matmul_validate(d, rescale != nullptr, &path, &bn));
    // Path 5 (B rows not 16-byte multiples, e.g. 1000 classes) pads B into a buffer of the
    // plan's own; here those shapes take the direct kernel instead (path 2), which keeps
    // nothing per call but the error word.
    if (path == 5) path = 2;
    if (rescale && rescale->channels > kMaxRescaleChannels)
        return fail(TB_ERR_INVALID_ARGUMENT, "tb_matmul_i8_noalloc: %d rescale channels exceed the scratch limit %d",
                    rescale->channels, kMaxRescaleChannels);
    if (d->a_zp != 0 && static_cast<long long>(d->n) * d->w > kMaxColterm)
        return fail(TB_ERR_INVALID_ARGUMENT, "tb_matmul_i8_noalloc: n*w = %lld exceeds the scratch limit %lld",
                    static_cast<long long>(d->n) * d->w, kMaxColterm);
    int dev = 0;
    TB_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxDevices) return fail(TB_ERR_INVALID_ARGUMENT, "device %d out of range", dev);
    DeviceSetup su;
    TB_TRY(device_setup(dev, &su));
    cudaStream_t st = static_cast<cudaStream_t>(stream_);

    // A context and a plan on the stack whose device pointers all point into the array.
    tb_context ctx;
    ctx.device = dev;
    ctx.num_sms = su.num_sms;
    ctx.dev_err = reinterpret_cast<uint32_t*>(su.scratch);
    ctx.timeout_cycles = su.timeout_cycles;
    tb_matmul_plan plan;
    plan.ctx = &ctx;
    plan.d = *d;
    plan.path = path;
    plan.bn = bn;
    std::vector<int32_t> blob, sr_blob;  // host copies stay alive until the call synchronizes
    if (rescale) {
        TB_TRY(prepare_rescale(rescale, TB_DT_INT32, d->w, &plan.rs, &blob));
        // the small-range epilogue constants (as tb_matmul_plan_create makes them)
        const long long bound = static_cast<long long>(d->c) * (128 + std::abs(d->a_zp)) * (128 + std::abs(d->b_zp));
        prepare_small_range(*rescale, plan.rs, bound, &plan.sr, &sr_blob);
        if (blob.size() + sr_blob.size() > kMaxBlobWords)
            return fail(TB_ERR_INVALID_ARGUMENT, "tb_matmul_i8_noalloc: %d rescale channels exceed the scratch limit",
                        rescale->channels);
        int32_t* dev_blob = reinterpret_cast<int32_t*>(su.scratch + kBlobOffset);
        TB_CUDA(cudaMemcpyAsync(dev_blob, blob.data(), sizeof(int32_t) * blob.size(), cudaMemcpyHostToDevice, st));
        place_rescale(&plan.rs, dev_blob);
        if (plan.sr.ok) {
            int32_t* dev_sr = dev_blob + blob.size();
            TB_CUDA(cudaMemcpyAsync(dev_sr, sr_blob.data(), sizeof(int32_t) * sr_blob.size(), cudaMemcpyHostToDevice,
                                    st));
            place_small_range(&plan.sr, dev_sr, rescale->channels);
        }
    }
    if (path == 0 && d->a_zp != 0) plan.d_colterm = reinterpret_cast<int32_t*>(su.scratch + kColtermOffset);
    // The array keeps the previous call's contents: the error word starts at zero.
    TB_CUDA(cudaMemsetAsync(su.scratch, 0, 8, st));
    TB_TRY(tb_matmul_plan_run(&plan, a, b, out, stream_));
    // Data-dependent errors (RESCALE ranges) are reported by this call itself.
    uint32_t word = 0;
    TB_CUDA(cudaMemcpyAsync(&word, su.scratch, sizeof word, cudaMemcpyDeviceToHost, st));
    TB_CUDA(cudaStreamSynchronize(st));
    plan.rs.d_blob = nullptr;  // nothing owned
    plan.sr.d_blob = nullptr;
    if (word & DEV_ERR_TIMEOUT) return fail(TB_ERR_TIMEOUT, "a device wait timed out");
    if (word) return fail(TB_ERR_GRAPH, "apply_scale: value out of range for the shift, or result exceeds int32");
    return TB_OK;
}
