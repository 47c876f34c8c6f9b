// gemm_noalloc.cu -- a projection GEMM entry point that allocates nothing.
//
// hllm_b200_gemm keeps its stream-K scratch (F32 partial tiles) in device
// memory that the library allocates on first use.  Some callers cannot let a
// library allocate device memory: a serving process that fixes its
// device-memory budget when it starts and admits every request against it
// (hLLM's worker reserves each request's bytes before running it,
// cpp/src/worker/control_service.cpp:391-461, so a buffer allocated later is
// outside the accounting and can fail under load), and hosts that own all
// device memory of a plugin.  This variant's scratch is a file-scope static
// __device__ array of a fixed maximum size, part of the library image: every
// GPU that loads the library holds it until the process exits.
//
// Set-up: the first call on a device, with that device current, resolves the
// array's device address with cudaGetSymbolAddress (the array's name in host
// code is only a host-side stand-in).  That first call should come before any
// stream capture on the device.
//
// Sharing: every call on a device uses the same array, which keeps the last
// call's contents.  Each call rewrites all of the scratch it reads, so nothing
// has to start at zero, except the status word, which is cleared per call.
// Calls whose GPU work overlaps (for example on two streams) race on the array
// and must not be issued.
#include <cuda_runtime.h>

#include <map>
#include <mutex>
#include <string>

#include "common.cuh"
#include "gemm.cuh"
#include "hllm_b200.h"

namespace hb {
void set_last_error(const std::string& message);  // stage.cu
}

namespace {

// 32 MiB of F32 partial tiles: enough for the stream-K splits of decode-width
// projections (up to 64 tokens per tile, gate/up pairs included, at 148 CTAs);
// larger stream-K plans are rejected.  Direct plans (at least two tiles per
// SM) need no partials.
constexpr size_t kNoAllocSlotFloats = size_t{8} << 20;

__device__ __align__(256) float g_noalloc_slots[kNoAllocSlotFloats];
__device__ __align__(256) uint32_t g_noalloc_status[64];

struct DevicePointers {
  float* slots = nullptr;
  uint32_t* status = nullptr;
  int sm_count = 0;
};

std::mutex g_mutex;
std::map<int, DevicePointers> g_pointers;

hllm_b200_status fail(hllm_b200_status code, const std::string& message) {
  hb::set_last_error(message);
  return code;
}

// Resolves the static arrays' device addresses for the current device (once).
hllm_b200_status pointers_for_current_device(DevicePointers* out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(HLLM_B200_INTERNAL, cudaGetErrorString(e));
  std::scoped_lock lock(g_mutex);
  auto it = g_pointers.find(dev);
  if (it == g_pointers.end()) {
    DevicePointers p;
    e = cudaGetSymbolAddress(reinterpret_cast<void**>(&p.slots), g_noalloc_slots);
    if (e == cudaSuccess) e = cudaGetSymbolAddress(reinterpret_cast<void**>(&p.status), g_noalloc_status);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&p.sm_count, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess)
      return fail(HLLM_B200_INTERNAL, std::string("static scratch set-up: ") + cudaGetErrorString(e));
    it = g_pointers.emplace(dev, p).first;
  }
  *out = it->second;
  return HLLM_B200_OK;
}

}  // namespace

extern "C" hllm_b200_status hllm_b200_gemm_noalloc(const void* w, uint64_t m, uint64_t k_pad,
                                                   uint32_t pair, uint64_t second_row,
                                                   const void* x, uint64_t n, uint32_t epilogue,
                                                   void* y, uint64_t ldy, uint32_t bn,
                                                   uint32_t grid, void* stream) {
  if (!w || !x || !y || m == 0 || n == 0 || k_pad == 0 || k_pad % 64 != 0 || epilogue > 3 ||
      (pair != 1 && pair != 2) || (pair == 2) != (epilogue == 3))
    return fail(HLLM_B200_INVALID_REQUEST, "invalid GEMM arguments");
  DevicePointers dp;
  hllm_b200_status st = pointers_for_current_device(&dp);
  if (st != HLLM_B200_OK) return st;
  hb::GemmWeight gw{};
  const int rows_total = pair == 2 ? static_cast<int>(second_row + m) : static_cast<int>(m);
  if (!hb::gemm_make_weight(&gw, w, rows_total, static_cast<int>(m), static_cast<int>(k_pad),
                            static_cast<int>(pair), static_cast<int>(second_row)))
    return fail(HLLM_B200_INTERNAL, "tensor map creation failed");
  hb::GemmInput gx{};
  if (!hb::gemm_make_input(&gx, x, static_cast<int>(n), static_cast<int>(k_pad),
                           static_cast<int>(k_pad)))
    return fail(HLLM_B200_INTERNAL, "tensor map creation failed");
  const hb::GemmPlan plan = hb::gemm_plan(gw, static_cast<int>(n), dp.sm_count,
                                          static_cast<int>(bn), static_cast<int>(grid));
  const size_t need = hb::gemm_slot_floats(plan, static_cast<int>(pair));
  if (need > kNoAllocSlotFloats)
    return fail(HLLM_B200_RESOURCE_EXHAUSTED,
                "GEMM split needs " + std::to_string(need * 4) +
                    " bytes of partial sums; the allocation-free entry point holds at most " +
                    std::to_string(kNoAllocSlotFloats * 4) +
                    " (use fewer CTAs, fewer tokens per call, or hllm_b200_gemm)");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemsetAsync(dp.status, 0, sizeof(uint32_t), s);
  hb::GemmSlots slots{};
  if (e == cudaSuccess)
    e = hb::gemm_launch(gw, gx, static_cast<int>(n), plan, static_cast<int>(epilogue), y,
                        static_cast<int>(ldy), dp.slots, &slots, dp.status, s);
  if (e == cudaSuccess && plan.stream_k)
    e = hb::gemm_finish_launch(slots, static_cast<int>(n), static_cast<int>(epilogue), y,
                               static_cast<int>(ldy), s);
  if (e != cudaSuccess)
    return fail(e == cudaErrorInvalidValue ? HLLM_B200_INVALID_REQUEST : HLLM_B200_INTERNAL,
                cudaGetErrorString(e));
  return HLLM_B200_OK;
}
