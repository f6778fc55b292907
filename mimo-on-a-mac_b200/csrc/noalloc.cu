// mimo_moe_experts_static: the small-batch expert products with their scratch in a fixed device array.
//
// Some callers cannot allocate device memory at the point where they run the MoE block: an inference
// runtime that hands this library only its activations and weights (with no allocator hook), code that
// runs inside a preallocated memory arena it must not grow, or a host process that is not allowed to
// call cudaMalloc at all.  For them this entry point keeps its scratch - the f16 copy of x, the SwiGLU
// output h and the per-route float partials - in one file-scope __device__ array instead of a
// caller-provided workspace.  Every GPU that loads the library holds that array (kScratchBytes) until
// the process exits.
//
// Set-up: the device address of the array is looked up once per device and CUDA context
// (cudaGetSymbolAddress with that device current), on the first call made there; a later call in a new
// context of the same device (after cudaDeviceReset, say) looks it up again, because the module and
// its array are loaded afresh.  Make that first call before any stream capture begins.  Calls share the
// array and each call overwrites it, so calls whose work overlaps on the GPU (two streams, or two
// threads) race; serialise them on one stream.  No part of the scratch has to start at zero: for valid
// route tables each call writes every scratch word before it reads it, and a route row outside [0, M)
// sets MIMO_ERANGE and reads row 0 instead of stale rows.
//
// Kernels: the mma.sync (f16 tensor core, CUDA-core e2m1 decode) decode kernels, not the tcgen05
// kernels of mimo_moe_experts (those need workspace for their activation term matrices).  The results
// therefore agree with mimo_moe_experts within the output tolerance, not bit for bit.
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"
#include "kernels.h"

namespace {

// Limits of this entry point: M <= 8 rows, U*R <= 512 route slots, H <= 4096, I <= 2048.
constexpr int kMaxRows = 8;
constexpr int kMaxSlots = 512;
constexpr int kMaxHidden = 4096;
constexpr int kMaxInter = 2048;
constexpr size_t kX16Bytes = (size_t)kMaxRows * kMaxHidden * 2;    //  64 KiB
constexpr size_t kH16Bytes = (size_t)kMaxSlots * kMaxInter * 2;    //   2 MiB
constexpr size_t kPartBytes = (size_t)kMaxSlots * kMaxHidden * 4;  //   8 MiB
constexpr size_t kScratchBytes = kX16Bytes + kH16Bytes + kPartBytes;

static __device__ __align__(256) unsigned char g_expert_scratch[kScratchBytes];

std::mutex g_mu;
struct ScratchAddr {
  void* ctx = nullptr;  // the CUDA context the address belongs to
  void* ptr = nullptr;
};
ScratchAddr g_scratch[128];

// The current CUDA context (driver handle), or null when it cannot be queried.
void* current_context() {
  static PFN_cuCtxGetCurrent_v4000 fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &p, 4000, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      p = nullptr;
    return reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(p);
  }();
  CUcontext c = nullptr;
  if (!fn || fn(&c) != CUDA_SUCCESS) return nullptr;
  return c;
}

}  // namespace

extern "C" {

size_t mimo_moe_experts_static_scratch_bytes(void) { return kScratchBytes; }

int mimo_moe_experts_static(const uint16_t* x, const mimo_moe_pools* pools, const int32_t* uslot,
                            const int32_t* urows, const int32_t* ucnt, const float* uw,
                            const int32_t* num_unique, int32_t U, int32_t R, const int32_t* gather_idx,
                            int32_t topk, int32_t M, int32_t pairs_rounding, uint16_t* y, int32_t* status,
                            void* stream) {
  using namespace mimo;
  if (!x || !pools || !uslot || !urows || !ucnt || !uw || !y || U < 1 || R < 1 || R > 8 || M < 1 ||
      (gather_idx && (topk < 1 || topk > 64)))
    return MIMO_EINVAL;
  if (!pools->gate_w || !pools->gate_s || !pools->up_w || !pools->up_s || !pools->down_w ||
      !pools->down_s || pools->num_slots < 1 || pools->hidden < 2048 || pools->inter < 2048 ||
      pools->hidden % 2048 || pools->inter % 2048)
    return MIMO_EINVAL;
  // Sizes beyond the fixed scratch are refused outright.
  if (M > kMaxRows || (int64_t)U * R > kMaxSlots || pools->hidden > kMaxHidden || pools->inter > kMaxInter)
    return MIMO_ERANGE;

  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= 128) return MIMO_ECUDA;
  void* base = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    void* ctx = current_context();
    ScratchAddr& a = g_scratch[dev];
    if (a.ptr == nullptr || ctx == nullptr || a.ctx != ctx) {
      void* p = nullptr;
      e = cudaGetSymbolAddress(&p, g_expert_scratch);
      if (e != cudaSuccess || p == nullptr) return MIMO_ECUDA;
      a.ptr = p;
      a.ctx = ctx;
    }
    base = a.ptr;
  }
  uint8_t* b = static_cast<uint8_t*>(base);
  __half* x16 = reinterpret_cast<__half*>(b);
  __half* h16 = reinterpret_cast<__half*>(b + kX16Bytes);
  float* part = reinterpret_cast<float*>(b + kX16Bytes + kH16Bytes);

  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int H = pools->hidden, I = pools->inter;
  int sms = 148;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) sms = 148;

  if ((e = launch_to_f16(x, x16, (size_t)M * H, status, st)) != cudaSuccess) return MIMO_ECUDA;
  ExpertParams p{};
  p.w[0] = reinterpret_cast<const uint8_t*>(pools->gate_w);
  p.s[0] = pools->gate_s;
  p.w[1] = reinterpret_cast<const uint8_t*>(pools->up_w);
  p.s[1] = pools->up_s;
  p.S = pools->num_slots;
  p.N = I;
  p.K = H;
  p.tiles = I / 16;
  p.unit_slot = uslot;
  p.unit_p0 = nullptr;
  p.p0_stride = R;
  p.unit_cnt = ucnt;
  p.num_units = num_unique;
  p.units_cap = U;
  p.rtok = urows;
  p.bsrc = x16;
  p.brows = M;
  p.h_out = h16;
  p.status = status;
  if ((e = launch_expert_tiles(p, 0, sms, st)) != cudaSuccess) return MIMO_ECUDA;
  ExpertParams q = p;
  q.w[0] = reinterpret_cast<const uint8_t*>(pools->down_w);
  q.s[0] = pools->down_s;
  q.w[1] = nullptr;
  q.s[1] = nullptr;
  q.N = H;
  q.K = I;
  q.tiles = H / 16;
  q.rtok = nullptr;
  q.bsrc = h16;
  q.brows = 0;
  q.h_out = nullptr;
  q.rw = uw;
  q.part_out = part;
  q.pairs_rounding = pairs_rounding;
  if ((e = launch_expert_tiles(q, 1, sms, st)) != cudaSuccess) return MIMO_ECUDA;
  if ((e = launch_combine_decode(part, gather_idx, urows, ucnt, num_unique, U, R, M, topk, H, y, status, st)) !=
      cudaSuccess)
    return MIMO_ECUDA;
  return MIMO_OK;
}

}  // extern "C"
