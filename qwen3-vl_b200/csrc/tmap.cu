// TMA tensor-map construction (host side) shared by the GEMM kernels.
#include <mutex>
#include <unordered_map>

#include "common.cuh"

namespace q3 {

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// cuTensorMapEncodeTiled through the runtime's driver entry point, so the
// library does not link libcuda directly.
static EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

int make_tmap_2d(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int box_rows,
                 int box_cols) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return fail(Q3_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  if (box_cols * 2 != 128 || box_rows < 1 || box_rows > 256)
    return fail(Q3_ERR_INVALID, "tensor map box %dx%d unsupported", box_rows, box_cols);
  if (!aligned(base, 16) || (cols * 2) % 16 != 0)
    return fail(Q3_ERR_INVALID, "tensor map base/row stride must be 16-byte aligned");
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims,
                   strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(Q3_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return Q3_OK;
}

int make_tmap_3d_rows128(CUtensorMap* map, const void* base, int64_t rows, int64_t planes,
                         int64_t plane_stride_elems, int box_rows) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return fail(Q3_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  if (box_rows < 1 || box_rows > 256 || rows < 1 || planes < 1)
    return fail(Q3_ERR_INVALID, "3-D tensor map: bad rows/planes/box");
  if (!aligned(base, 16) || (plane_stride_elems * 2) % 16 != 0)
    return fail(Q3_ERR_INVALID, "3-D tensor map: base/plane stride must be 16-byte aligned");
  cuuint64_t dims[3] = {128, (cuuint64_t)rows, (cuuint64_t)planes};
  cuuint64_t strides[2] = {256, (cuuint64_t)plane_stride_elems * 2};
  cuuint32_t box[3] = {64, (cuuint32_t)box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims,
                   strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(Q3_ERR_CUDA, "cuTensorMapEncodeTiled (3-D) failed (%d)", (int)r);
  return Q3_OK;
}

int make_tmap_wblocks(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int box_rows,
                      int depth) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return fail(Q3_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  if (cols % 64 != 0 || box_rows < 1 || box_rows > 256 || depth < 1 || depth > 256)
    return fail(Q3_ERR_INVALID, "weight-block tensor map: bad shape");
  if (!aligned(base, 16))
    return fail(Q3_ERR_INVALID, "weight-block tensor map: base must be 16-byte aligned");
  cuuint64_t dims[3] = {64, (cuuint64_t)rows, (cuuint64_t)(cols / 64)};
  cuuint64_t strides[2] = {(cuuint64_t)cols * 2, 128};
  cuuint32_t box[3] = {64, (cuuint32_t)box_rows, (cuuint32_t)depth};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims,
                   strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(Q3_ERR_CUDA, "cuTensorMapEncodeTiled (weight blocks) failed (%d)", (int)r);
  return Q3_OK;
}

namespace {
struct TmapKey {
  const void* p;
  int64_t rows, cols;
  int box_rows, box_cols;
  bool operator==(const TmapKey& o) const {
    return p == o.p && rows == o.rows && cols == o.cols && box_rows == o.box_rows &&
           box_cols == o.box_cols;
  }
};
struct TmapKeyHash {
  size_t operator()(const TmapKey& k) const {
    return std::hash<const void*>()(k.p) ^ (size_t)(k.rows * 1315423911ll) ^
           (size_t)(k.cols * 2654435761ll) ^ ((size_t)k.box_rows << 20) ^ (size_t)k.box_cols;
  }
};
}  // namespace

int cached_tmap_2d(CUtensorMap* out, const void* base, int64_t rows, int64_t cols, int box_rows,
                   int box_cols) {
  static std::mutex mu;
  static std::unordered_map<TmapKey, CUtensorMap, TmapKeyHash> cache;
  TmapKey key{base, rows, cols, box_rows, box_cols};
  {
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find(key);
    if (it != cache.end()) {
      *out = it->second;
      return Q3_OK;
    }
  }
  int rc = make_tmap_2d(out, base, rows, cols, box_rows, box_cols);
  if (rc != Q3_OK) return rc;
  std::lock_guard<std::mutex> lock(mu);
  if (cache.size() > 4096) cache.clear();
  cache[key] = *out;
  return Q3_OK;
}

}  // namespace q3
