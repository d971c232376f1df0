// Host-side TMA tensor-map encoding and ABI-wide helpers.
#include <cudaTypedefs.h>

#include "common.cuh"

std::mutex& tsds_host_cache_lock() {
  static std::mutex m;
  return m;
}

// The driver's tensor-map encoder, looked up once (any thread may be first;
// a second lookup finds the same entry point).
static std::atomic<PFN_cuTensorMapEncodeTiled_v12000> g_encode_tiled{nullptr};

static PFN_cuTensorMapEncodeTiled_v12000 load_encode_tiled() {
  PFN_cuTensorMapEncodeTiled_v12000 f = g_encode_tiled.load(std::memory_order_acquire);
  if (f) return f;
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
      q != cudaDriverEntryPointSuccess || fn == nullptr) {
    cudaGetLastError();
    return nullptr;
  }
  f = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  g_encode_tiled.store(f, std::memory_order_release);
  return f;
}

int tsds_make_tmap_2d_bf16(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
                           uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
                           int swizzle_128b) {
  const PFN_cuTensorMapEncodeTiled_v12000 encode = load_encode_tiled();
  if (!encode) return TSDS_E_DEVICE;
  if (!tsds_aligned16(base) || (row_stride_bytes % 16) != 0) return TSDS_E_ALIGN;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides,
                              box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                              swizzle_128b ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? TSDS_OK : TSDS_E_INVALID;
}

extern "C" const char* tsds_status_string(int status) {
  switch (status) {
    case TSDS_OK: return "ok";
    case TSDS_E_INVALID: return "invalid argument or shape";
    case TSDS_E_ALIGN: return "pointer or leading dimension not 16-byte aligned";
    case TSDS_E_LAUNCH: return "kernel launch failed";
    case TSDS_E_WORKSPACE: return "workspace too small";
    case TSDS_E_TIMEOUT: return "device-side bounded wait timed out";
    case TSDS_E_UNSUPPORTED: return "unsupported configuration";
    case TSDS_E_DEVICE: return "device / driver query failed";
    case TSDS_E_SCRATCH_LIMIT: return "request larger than the built-in scratch area";
    case TSDS_E_RUNTIME: return "CUDA runtime call (allocation / IPC) failed";
    case TSDS_E_INDEX: return "KV pool row outside the pool (table entry)";
    default: return "unknown status";
  }
}

extern "C" int tsds_abi_version(void) { return 1; }

static std::atomic<long long> g_launches{0};
void tsds_count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }
extern "C" int64_t tsds_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

static std::atomic<int> g_pdl{1};
int tsds_pdl_enabled() { return g_pdl; }
extern "C" void tsds_set_pdl(int on) { g_pdl = on ? 1 : 0; }
