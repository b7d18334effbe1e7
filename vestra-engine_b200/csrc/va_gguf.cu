// GGUF model files (the reference's crates/da-gguf): a host reader over a
// read-only mapping of the file, and device kernels that turn a tensor's stored
// bytes (F32, F16 or Q8_0 blocks) into F32 or bf16 on the GPU, with the rank-2
// transpose of weights_from_gguf (engine.rs:110-126) fused in.
//
// Container, little-endian (reader.rs:213-266):
//   "GGUF", u32 version (2 or 3), u64 tensor_count, u64 kv_count,
//   kv_count x {string key, u32 vtype, value},
//   tensor_count x {string name, u32 n_dims, u64 dims[n_dims] innermost first,
//                   u32 dtype, u64 offset},
//   zero padding up to `general.alignment` (32 unless a u32 key sets it),
//   data: tensor i starts at data_start + offset_i.
// A string is a u64 byte count and the bytes, decoded as UTF-8 with invalid
// sequences replaced by U+FFFD (String::from_utf8_lossy).
//
// Q8_0 (q8_0.rs:10-33): blocks of 32 values, 34 bytes each: an IEEE half scale d
// then 32 int8 quants q; value j = f32(d) * f32(q[j]).  The product of an 11-bit
// and an 8-bit significand is exact in F32, so the device result is bit-identical
// to the reference's host loop.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cerrno>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include <cuda_fp16.h>

#include "../../include/vestra_attn.h"
#include "va_internal.h"

namespace {

constexpr uint32_t kGgmlF32 = 0, kGgmlF16 = 1, kGgmlQ8_0 = 8;  // reader.rs:52-55
constexpr int kQk8_0 = 32, kQ8BlockBytes = 34;

struct Meta {
  std::string key;
  int kind = 0;                     // VA_META_*
  uint64_t bits = 0;                // scalar value (32-bit kinds in the low word)
  std::string s;                    // VA_META_STR
  std::vector<uint32_t> words;      // VA_META_ARR_{U32,I32,F32}
  std::vector<std::string> strs;    // VA_META_ARR_STR
};

struct TensorInfo {
  std::string name;
  std::vector<uint64_t> dims;  // innermost first, as stored
  uint32_t dtype = 0;
  uint64_t offset = 0;
};

thread_local std::string t_err;

int gerr(int code, std::string msg) {
  t_err = std::move(msg);
  return code;
}

int malformed(const std::string& what) { return gerr(VA_ERR_FORMAT, "malformed: " + what); }

// String::from_utf8_lossy: each maximal ill-formed subsequence becomes U+FFFD.
std::string utf8_lossy(const uint8_t* b, size_t n) {
  static const char kRepl[] = "\xEF\xBF\xBD";
  std::string out;
  out.reserve(n);
  size_t i = 0;
  while (i < n) {
    const uint8_t c = b[i];
    if (c < 0x80) {
      out.push_back(static_cast<char>(c));
      ++i;
      continue;
    }
    int len = 0;
    uint8_t lo = 0x80, hi = 0xBF;  // range of the second byte
    if (c >= 0xC2 && c <= 0xDF) {
      len = 2;
    } else if (c == 0xE0) {
      len = 3, lo = 0xA0;
    } else if ((c >= 0xE1 && c <= 0xEC) || c == 0xEE || c == 0xEF) {
      len = 3;
    } else if (c == 0xED) {
      len = 3, hi = 0x9F;
    } else if (c == 0xF0) {
      len = 4, lo = 0x90;
    } else if (c >= 0xF1 && c <= 0xF3) {
      len = 4;
    } else if (c == 0xF4) {
      len = 4, hi = 0x8F;
    }
    if (len == 0) {
      out += kRepl;
      ++i;
      continue;
    }
    size_t j = 1;
    while (j < static_cast<size_t>(len) && i + j < n) {
      const uint8_t d = b[i + j];
      const bool ok = (j == 1) ? (d >= lo && d <= hi) : (d >= 0x80 && d <= 0xBF);
      if (!ok) break;
      ++j;
    }
    if (j == static_cast<size_t>(len)) {
      out.append(reinterpret_cast<const char*>(b + i), j);
    } else {
      out += kRepl;
    }
    i += j;
  }
  return out;
}

struct Cursor {
  const uint8_t* b;
  size_t n;
  size_t p = 0;
  bool take(size_t k, const uint8_t** out) {
    if (k > n - p) return false;
    *out = b + p;
    p += k;
    return true;
  }
  template <class T>
  bool get(T* v) {
    const uint8_t* q;
    if (!take(sizeof(T), &q)) return false;
    std::memcpy(v, q, sizeof(T));
    return true;
  }
  bool str(std::string* s) {
    uint64_t k;
    const uint8_t* q;
    if (!get(&k) || k > n - p || !take(static_cast<size_t>(k), &q)) return false;
    *s = utf8_lossy(q, static_cast<size_t>(k));
    return true;
  }
};

uint32_t f32_bits(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  return u;
}

// read_kv_value (reader.rs:86-208).  Returns VA_OK with *skipped set for the
// spec-valid array element types the reader does not keep.
int read_value(Cursor& c, uint32_t vtype, Meta* m, bool* skipped) {
  *skipped = false;
  const uint8_t* q;
  switch (vtype) {
    case 0: case 1: {  // uint8, int8: the byte, zero-extended (`[0] as u32` / `as i32`)
      if (!c.take(1, &q)) return malformed("eof");
      m->kind = vtype == 0 ? VA_META_U32 : VA_META_I32;
      m->bits = q[0];
      return VA_OK;
    }
    case 2: {
      uint16_t v;
      if (!c.get(&v)) return malformed("eof");
      m->kind = VA_META_U32, m->bits = v;
      return VA_OK;
    }
    case 3: {  // int16, sign-extended
      int16_t v;
      if (!c.get(&v)) return malformed("eof");
      m->kind = VA_META_I32, m->bits = static_cast<uint32_t>(static_cast<int32_t>(v));
      return VA_OK;
    }
    case 4: case 5: case 6: {
      uint32_t v;
      if (!c.get(&v)) return malformed("eof");
      m->kind = vtype == 4 ? VA_META_U32 : vtype == 5 ? VA_META_I32 : VA_META_F32;
      m->bits = v;
      return VA_OK;
    }
    case 7: {
      if (!c.take(1, &q)) return malformed("eof");
      m->kind = VA_META_BOOL, m->bits = q[0] != 0;
      return VA_OK;
    }
    case 8:
      if (!c.str(&m->s)) return malformed("eof");
      m->kind = VA_META_STR;
      return VA_OK;
    case 10: case 11: {  // uint64, int64 (kept as its bit pattern, `as u64`)
      uint64_t v;
      if (!c.get(&v)) return malformed("eof");
      m->kind = VA_META_U64, m->bits = v;
      return VA_OK;
    }
    case 12: {  // float64, narrowed to F32 (`as f32`, round to nearest even)
      double v;
      if (!c.get(&v)) return malformed("eof");
      m->kind = VA_META_F32, m->bits = f32_bits(static_cast<float>(v));
      return VA_OK;
    }
    case 9: {
      uint32_t elem;
      uint64_t count;
      if (!c.get(&elem) || !c.get(&count)) return malformed("eof");
      switch (elem) {
        case 4: case 5: case 6: {
          if (count > (c.n - c.p) / 4) return malformed("eof");
          m->kind = elem == 4 ? VA_META_ARR_U32 : elem == 5 ? VA_META_ARR_I32 : VA_META_ARR_F32;
          m->words.resize(static_cast<size_t>(count));
          if (!c.take(static_cast<size_t>(count) * 4, &q)) return malformed("eof");
          if (count) std::memcpy(m->words.data(), q, static_cast<size_t>(count) * 4);
          return VA_OK;
        }
        case 8: {
          m->kind = VA_META_ARR_STR;
          for (uint64_t i = 0; i < count; ++i) {
            std::string s;
            if (!c.str(&s)) return malformed("eof");
            m->strs.push_back(std::move(s));
          }
          return VA_OK;
        }
        case 0: case 1: case 2: case 3: case 7: case 10: case 11: case 12: {
          const uint64_t width = (elem == 0 || elem == 1 || elem == 7) ? 1 : (elem == 2 || elem == 3) ? 2 : 8;
          if (count > (c.n - c.p) / width) return malformed("eof");
          c.take(static_cast<size_t>(count * width), &q);
          *skipped = true;
          return VA_OK;
        }
        default:
          return malformed("array element type " + std::to_string(elem));
      }
    }
    default:
      return malformed("kv type " + std::to_string(vtype));
  }
}

const Meta* find_meta(const va_gguf* g, const char* key);
const TensorInfo* find_tensor(const va_gguf* g, const char* name);

}  // namespace

struct va_gguf {
  int fd = -1;
  const uint8_t* map = nullptr;
  size_t len = 0;
  uint32_t version = 0;
  uint64_t alignment = 32;
  size_t data_start = 0;
  std::vector<Meta> kv;
  std::vector<TensorInfo> tensors;
  ~va_gguf() {
    if (map) munmap(const_cast<uint8_t*>(map), len);
    if (fd >= 0) close(fd);
  }
};

namespace {

const Meta* find_meta(const va_gguf* g, const char* key) {
  for (const Meta& m : g->kv)
    if (m.key == key) return &m;  // the first entry of that key, like meta() (meta.rs:16-18)
  return nullptr;
}

const TensorInfo* find_tensor(const va_gguf* g, const char* name) {
  for (const TensorInfo& t : g->tensors)
    if (t.name == name) return &t;
  return nullptr;
}

// GgufFile::open's parse (reader.rs:213-266) over the mapped bytes.
int parse(va_gguf* g) {
  Cursor c{g->map, g->len};
  const uint8_t* q;
  if (!c.take(4, &q)) return malformed("eof");
  if (std::memcmp(q, "GGUF", 4) != 0) return gerr(VA_ERR_FORMAT, "bad magic");
  uint64_t tensor_count, kv_count;
  if (!c.get(&g->version)) return malformed("eof");
  if (g->version != 2 && g->version != 3)
    return gerr(VA_ERR_FORMAT, "unsupported gguf version " + std::to_string(g->version));
  if (!c.get(&tensor_count) || !c.get(&kv_count)) return malformed("eof");
  for (uint64_t i = 0; i < kv_count; ++i) {
    Meta m;
    uint32_t vtype;
    if (!c.str(&m.key) || !c.get(&vtype)) return malformed("eof");
    if (m.key == "general.alignment" && vtype == 4) {
      uint32_t a;
      if (!c.get(&a)) return malformed("eof");
      if (a == 0) return malformed("general.alignment is 0");
      g->alignment = a;
      m.kind = VA_META_U32, m.bits = a;
      g->kv.push_back(std::move(m));
      continue;
    }
    bool skipped;
    int rc = read_value(c, vtype, &m, &skipped);
    if (rc) return rc;
    if (!skipped) g->kv.push_back(std::move(m));
  }
  for (uint64_t i = 0; i < tensor_count; ++i) {
    TensorInfo t;
    uint32_t n_dims;
    if (!c.str(&t.name) || !c.get(&n_dims)) return malformed("eof");
    if (n_dims > (c.n - c.p) / 8) return malformed("eof");
    t.dims.resize(n_dims);
    for (uint32_t d = 0; d < n_dims; ++d) c.get(&t.dims[d]);
    if (!c.get(&t.dtype) || !c.get(&t.offset)) return malformed("eof");
    g->tensors.push_back(std::move(t));
  }
  const uint64_t pad = (g->alignment - (c.p % g->alignment)) % g->alignment;
  g->data_start = c.p + static_cast<size_t>(pad);
  return VA_OK;
}

bool mul_ok(uint64_t a, uint64_t b, uint64_t* out) {
  if (a != 0 && b > UINT64_MAX / a) return false;
  *out = a * b;
  return true;
}

// The checks of tensor_f32 (reader.rs:279-349), in its order.
int check_tensor(const va_gguf* g, const TensorInfo& t, uint64_t* numel, uint64_t* base, uint64_t* bytes) {
  // The element count wraps at 2^64, as the reference's `product()` of usize does
  // in a release build; the byte range below is checked without wrapping.
  uint64_t n = 1;
  for (uint64_t d : t.dims) n *= d;
  const uint64_t b = static_cast<uint64_t>(g->data_start) + t.offset;
  const bool base_ok = b >= t.offset;
  uint64_t nb = 0;
  bool size_ok = true;
  switch (t.dtype) {
    case kGgmlF32: size_ok = mul_ok(n, 4, &nb); break;
    case kGgmlF16: size_ok = mul_ok(n, 2, &nb); break;
    case kGgmlQ8_0:
      if (n % kQk8_0 != 0)
        return malformed("tensor '" + t.name + "' has " + std::to_string(n) +
                         " elements, not a multiple of block size 32 (QK8_0)");
      size_ok = mul_ok(n / kQk8_0, kQ8BlockBytes, &nb);
      break;
    default:
      return gerr(VA_ERR_DTYPE, "unsupported dtype " + std::to_string(t.dtype));
  }
  const uint64_t end = b + nb;
  if (!base_ok || !size_ok || end < b || end > g->len)
    return malformed("tensor '" + t.name + "' data out of bounds: [" + std::to_string(b) + ", " +
                     (base_ok && size_ok && end >= b ? std::to_string(end) : std::string("overflow")) +
                     ") exceeds file size " + std::to_string(g->len));
  *numel = n;
  *base = b;
  *bytes = nb;
  return VA_OK;
}

// ------------------------------------------------------------------ device kernels
__device__ __forceinline__ float load1(const uint8_t* __restrict__ src, uint32_t dtype, int64_t e) {
  if (dtype == kGgmlF32) return reinterpret_cast<const float*>(src)[e];
  if (dtype == kGgmlF16) return __half2float(reinterpret_cast<const __half*>(src)[e]);
  const uint8_t* blk = src + (e >> 5) * kQ8BlockBytes;
  const float d = __half2float(*reinterpret_cast<const __half*>(blk));
  return d * static_cast<float>(static_cast<int8_t>(blk[2 + (e & 31)]));
}

// Eight consecutive values from e0 (a multiple of 8, e0 + 8 <= n).  The source
// buffer starts 256-byte aligned, so F32 runs are 32-byte and F16 runs 16-byte
// aligned; a Q8_0 run lies inside one block at an even offset.
__device__ __forceinline__ void load8(const uint8_t* __restrict__ src, uint32_t dtype, int64_t e0, float v[8]) {
  if (dtype == kGgmlF32) {
    const float4 a = reinterpret_cast<const float4*>(src)[e0 / 4];
    const float4 b = reinterpret_cast<const float4*>(src)[e0 / 4 + 1];
    v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
  } else if (dtype == kGgmlF16) {
    const uint4 u = *reinterpret_cast<const uint4*>(src + 2 * e0);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
      v[2 * i] = f.x, v[2 * i + 1] = f.y;
    }
  } else {
    const uint8_t* blk = src + (e0 >> 5) * kQ8BlockBytes;
    const float d = __half2float(*reinterpret_cast<const __half*>(blk));
    const uint16_t* qp = reinterpret_cast<const uint16_t*>(blk + 2 + (e0 & 31));
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint16_t h = qp[i];
      v[2 * i] = d * static_cast<float>(static_cast<int8_t>(h & 0xff));
      v[2 * i + 1] = d * static_cast<float>(static_cast<int8_t>(h >> 8));
    }
  }
}

template <class T> __device__ __forceinline__ T cvt(float x);
template <> __device__ __forceinline__ float cvt<float>(float x) { return x; }
template <> __device__ __forceinline__ __nv_bfloat16 cvt<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }

__device__ __forceinline__ void store8(float* p, const float v[8]) {
  reinterpret_cast<float4*>(p)[0] = make_float4(v[0], v[1], v[2], v[3]);
  reinterpret_cast<float4*>(p)[1] = make_float4(v[4], v[5], v[6], v[7]);
}
__device__ __forceinline__ void store8(__nv_bfloat16* p, const float v[8]) {
  uint4 u;
  uint32_t* w = &u.x;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
    w[i] = *reinterpret_cast<const uint32_t*>(&h);
  }
  *reinterpret_cast<uint4*>(p) = u;
}

// dst[r*ld + c] = value(r*cols + c): one thread per eight stored values.
template <class OutT>
__global__ void __launch_bounds__(256) gguf_rows_kernel(const uint8_t* __restrict__ src, uint32_t dtype,
                                                        int64_t n, int64_t cols, int64_t ld, int vec_ok,
                                                        OutT* __restrict__ dst) {
  const int64_t e0 = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 8;
  if (e0 >= n) return;
  float v[8];
  const bool full = e0 + 8 <= n;
  if (full) {
    load8(src, dtype, e0, v);
  } else {
    for (int i = 0; i < 8; ++i) v[i] = e0 + i < n ? load1(src, dtype, e0 + i) : 0.f;
  }
  if (full && vec_ok) {
    const int64_t r = e0 / cols;
    store8(dst + r * ld + (e0 - r * cols), v);
    return;
  }
  for (int i = 0; i < 8 && e0 + i < n; ++i) {
    const int64_t e = e0 + i, r = e / cols;
    dst[r * ld + (e - r * cols)] = cvt<OutT>(v[i]);
  }
}

// dst[c*ld + r] = value(r*cols + c) through a 32x32 shared tile.
template <class OutT>
__global__ void __launch_bounds__(256) gguf_transpose_kernel(const uint8_t* __restrict__ src, uint32_t dtype,
                                                             int64_t rows, int64_t cols, int64_t ld,
                                                             OutT* __restrict__ dst) {
  __shared__ float tile[32][33];
  const int64_t c0 = static_cast<int64_t>(blockIdx.x) * 32;
  const int64_t row_tiles = (rows + 31) / 32;
  for (int64_t by = blockIdx.y; by < row_tiles; by += gridDim.y) {
    const int64_t r0 = by * 32;
    for (int i = threadIdx.y; i < 32; i += 8) {
      const int64_t r = r0 + i, c = c0 + threadIdx.x;
      if (r < rows && c < cols) tile[i][threadIdx.x] = load1(src, dtype, r * cols + c);
    }
    __syncthreads();
    for (int i = threadIdx.y; i < 32; i += 8) {
      const int64_t c = c0 + i, r = r0 + threadIdx.x;
      if (c < cols && r < rows) dst[c * ld + r] = cvt<OutT>(tile[threadIdx.x][i]);
    }
    __syncthreads();
  }
}

template <class OutT>
cudaError_t launch_convert_t(const uint8_t* src, uint32_t dtype, int64_t rows, int64_t cols, int64_t ld,
                             bool transpose, OutT* dst, cudaStream_t st) {
  if (rows <= 0 || cols <= 0) return cudaSuccess;
  if (!transpose) {
    const int64_t n = rows * cols;
    const bool aligned = (reinterpret_cast<uintptr_t>(dst) & 15) == 0;
    const int vec_ok = aligned && (ld == cols || (cols % 8 == 0 && ld % 8 == 0));
    const int64_t blocks = (n + 2047) / 2048;
    if (blocks > 0x7fffffff) return cudaErrorInvalidValue;
    gguf_rows_kernel<OutT><<<static_cast<unsigned>(blocks), 256, 0, st>>>(src, dtype, n, cols, ld, vec_ok, dst);
  } else {
    const int64_t col_tiles = (cols + 31) / 32, row_tiles = (rows + 31) / 32;
    if (col_tiles > 0x7fffffff) return cudaErrorInvalidValue;
    dim3 grid(static_cast<unsigned>(col_tiles), static_cast<unsigned>(row_tiles < 65535 ? row_tiles : 65535));
    gguf_transpose_kernel<OutT><<<grid, dim3(32, 8), 0, st>>>(src, dtype, rows, cols, ld, dst);
  }
  return cudaGetLastError();
}

}  // namespace

namespace va {

int gguf_tensor_ref(const va_gguf* g, const char* name, GgufTensorRef* out) {
  if (!g || !name || !out) return gerr(VA_ERR_INVALID, "null argument");
  const TensorInfo* t = find_tensor(g, name);
  if (!t) return gerr(VA_ERR_NOT_FOUND, std::string("tensor not found: ") + name);
  uint64_t n, base, bytes;
  int rc = check_tensor(g, *t, &n, &base, &bytes);
  if (rc) return rc;
  out->dtype = static_cast<int>(t->dtype);
  out->ndims = static_cast<int>(t->dims.size());
  for (int i = 0; i < 8; ++i)  // outer -> inner, the reversed stored order (reader.rs:300)
    out->shape[i] = i < out->ndims ? static_cast<int64_t>(t->dims[t->dims.size() - 1 - i]) : 1;
  out->numel = static_cast<int64_t>(n);
  out->data = g->map + base;
  out->bytes = static_cast<size_t>(bytes);
  return VA_OK;
}

const char* gguf_message() { return t_err.c_str(); }

cudaError_t launch_gguf_convert(const uint8_t* src, int dtype, int64_t rows, int64_t cols, int64_t ld,
                                bool transpose, bool out_bf16, void* dst, cudaStream_t st) {
  const uint32_t dt = static_cast<uint32_t>(dtype);
  if (dt != kGgmlF32 && dt != kGgmlF16 && dt != kGgmlQ8_0) return cudaErrorInvalidValue;
  if (out_bf16)
    return launch_convert_t(src, dt, rows, cols, ld, transpose, static_cast<__nv_bfloat16*>(dst), st);
  return launch_convert_t(src, dt, rows, cols, ld, transpose, static_cast<float*>(dst), st);
}

GgufStager::~GgufStager() {
  if (stream_) cudaStreamSynchronize(stream_);
  release();
  if (stream_) cudaStreamDestroy(stream_);
  for (cudaEvent_t& e : ev_)
    if (e) cudaEventDestroy(e);
}

void GgufStager::release() {
  for (int s = 0; s < 2; ++s) {
    if (pinned_[s]) cudaFreeHost(pinned_[s]);
    if (raw_[s]) cudaFree(raw_[s]);
    pinned_[s] = nullptr, raw_[s] = nullptr;
    used_[s] = false;
  }
  cap_ = 0;
}

cudaError_t GgufStager::reserve(size_t bytes) {
  if (!stream_) {
    cudaError_t e = cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking);
    if (e != cudaSuccess) return e;
    for (cudaEvent_t& ev : ev_)
      if ((e = cudaEventCreateWithFlags(&ev, cudaEventDisableTiming)) != cudaSuccess) return e;
  }
  if (bytes <= cap_) return cudaSuccess;
  cudaError_t e = cudaStreamSynchronize(stream_);
  if (e != cudaSuccess) return e;
  release();
  const size_t cap = (bytes + (1u << 20) - 1) & ~static_cast<size_t>((1u << 20) - 1);
  for (int s = 0; s < 2; ++s) {
    if ((e = cudaMallocHost(reinterpret_cast<void**>(&pinned_[s]), cap)) != cudaSuccess) return e;
    if ((e = cudaMalloc(reinterpret_cast<void**>(&raw_[s]), cap)) != cudaSuccess) return e;
  }
  cap_ = cap;
  return cudaSuccess;
}

cudaError_t GgufStager::convert(const GgufTensorRef& t, int64_t rows, int64_t cols, int64_t ld, bool transpose,
                                bool out_bf16, void* dst) {
  cudaError_t e = reserve(t.bytes);
  if (e != cudaSuccess) return e;
  const int s = slot_;
  slot_ ^= 1;
  // The copy engine may still read this slot's pinned bytes for the tensor before last.
  if (used_[s] && (e = cudaEventSynchronize(ev_[s])) != cudaSuccess) return e;
  std::memcpy(pinned_[s], t.data, t.bytes);
  if ((e = cudaMemcpyAsync(raw_[s], pinned_[s], t.bytes, cudaMemcpyHostToDevice, stream_)) != cudaSuccess) return e;
  if ((e = launch_gguf_convert(raw_[s], t.dtype, rows, cols, ld, transpose, out_bf16, dst, stream_)) != cudaSuccess)
    return e;
  used_[s] = true;
  uploaded += t.bytes;
  return cudaEventRecord(ev_[s], stream_);
}

cudaError_t GgufStager::zero(void* dst, size_t bytes) {
  cudaError_t e = reserve(0);
  return e != cudaSuccess ? e : cudaMemsetAsync(dst, 0, bytes, stream_);
}

cudaError_t GgufStager::finish() { return stream_ ? cudaStreamSynchronize(stream_) : cudaSuccess; }

}  // namespace va

// ------------------------------------------------------------------ C ABI
extern "C" {

const char* va_gguf_last_error(void) { return t_err.c_str(); }

int va_gguf_open(const char* path, va_gguf** out) {
  if (!path || !out) return gerr(VA_ERR_INVALID, "null argument");
  *out = nullptr;
  va_gguf* g = new (std::nothrow) va_gguf();
  if (!g) return gerr(VA_ERR_IO, "io: out of memory");
  g->fd = open(path, O_RDONLY | O_CLOEXEC);
  if (g->fd < 0) {
    const int err = errno;
    delete g;
    return gerr(VA_ERR_IO, std::string("io: ") + std::strerror(err) + ": " + path);
  }
  struct stat st;
  if (fstat(g->fd, &st) != 0) {
    const int err = errno;
    delete g;
    return gerr(VA_ERR_IO, std::string("io: ") + std::strerror(err));
  }
  g->len = static_cast<size_t>(st.st_size);
  if (g->len > 0) {
    void* m = mmap(nullptr, g->len, PROT_READ, MAP_PRIVATE, g->fd, 0);
    if (m == MAP_FAILED) {
      const int err = errno;
      g->len = 0;
      delete g;
      return gerr(VA_ERR_IO, std::string("io: ") + std::strerror(err));
    }
    g->map = static_cast<const uint8_t*>(m);
  }
  int rc = parse(g);
  if (rc) {
    delete g;
    return rc;
  }
  *out = g;
  return VA_OK;
}

void va_gguf_close(va_gguf* g) { delete g; }

int va_gguf_version(const va_gguf* g, uint32_t* version) {
  if (!g || !version) return gerr(VA_ERR_INVALID, "null argument");
  *version = g->version;
  return VA_OK;
}

int va_gguf_meta_count(const va_gguf* g, int64_t* n) {
  if (!g || !n) return gerr(VA_ERR_INVALID, "null argument");
  *n = static_cast<int64_t>(g->kv.size());
  return VA_OK;
}

int va_gguf_meta_entry(const va_gguf* g, int64_t i, const char** key, int64_t* key_len, int* kind) {
  if (!g || i < 0 || i >= static_cast<int64_t>(g->kv.size())) return gerr(VA_ERR_INVALID, "entry out of range");
  const Meta& m = g->kv[static_cast<size_t>(i)];
  if (key) *key = m.key.c_str();
  if (key_len) *key_len = static_cast<int64_t>(m.key.size());
  if (kind) *kind = m.kind;
  return VA_OK;
}

#define VA_META_GET(key_)                                                                  \
  if (!g || !(key_)) return gerr(VA_ERR_INVALID, "null argument");                        \
  const Meta* m = find_meta(g, key_);                                                      \
  if (!m) return gerr(VA_ERR_NOT_FOUND, std::string("metadata key not found: ") + (key_));

static int wrong_kind(const char* key) {
  return gerr(VA_ERR_NOT_FOUND, std::string("metadata key of another type: ") + key);
}

int va_gguf_meta_u32(const va_gguf* g, const char* key, uint32_t* out) {
  VA_META_GET(key)
  if (m->kind != VA_META_U32 && m->kind != VA_META_I32) return wrong_kind(key);
  if (out) *out = static_cast<uint32_t>(m->bits);
  return VA_OK;
}

int va_gguf_meta_i32(const va_gguf* g, const char* key, int32_t* out) {
  VA_META_GET(key)
  if (m->kind != VA_META_U32 && m->kind != VA_META_I32) return wrong_kind(key);
  if (out) *out = static_cast<int32_t>(static_cast<uint32_t>(m->bits));
  return VA_OK;
}

int va_gguf_meta_f32(const va_gguf* g, const char* key, float* out) {
  VA_META_GET(key)
  if (m->kind != VA_META_F32) return wrong_kind(key);
  const uint32_t b = static_cast<uint32_t>(m->bits);
  if (out) std::memcpy(out, &b, 4);
  return VA_OK;
}

int va_gguf_meta_u64(const va_gguf* g, const char* key, uint64_t* out) {
  VA_META_GET(key)
  if (m->kind != VA_META_U64) return wrong_kind(key);
  if (out) *out = m->bits;
  return VA_OK;
}

int va_gguf_meta_bool(const va_gguf* g, const char* key, int* out) {
  VA_META_GET(key)
  if (m->kind != VA_META_BOOL) return wrong_kind(key);
  if (out) *out = static_cast<int>(m->bits);
  return VA_OK;
}

int va_gguf_meta_str(const va_gguf* g, const char* key, const char** s, int64_t* len) {
  VA_META_GET(key)
  if (m->kind != VA_META_STR) return wrong_kind(key);
  if (s) *s = m->s.c_str();
  if (len) *len = static_cast<int64_t>(m->s.size());
  return VA_OK;
}

static int arr_words(const va_gguf* g, const char* key, bool want_i32, int want_kind, void* out, int64_t cap,
                     int64_t* count) {
  VA_META_GET(key)
  const bool ok = m->kind == want_kind || (want_i32 && m->kind == VA_META_ARR_U32);
  if (!ok) return wrong_kind(key);
  const int64_t n = static_cast<int64_t>(m->words.size());
  if (count) *count = n;
  if (out && cap > 0 && n > 0) std::memcpy(out, m->words.data(), static_cast<size_t>(n < cap ? n : cap) * 4);
  if (out && cap < n) return gerr(VA_ERR_CAPACITY, std::string("array longer than the buffer: ") + key);
  return VA_OK;
}

int va_gguf_meta_arr_u32(const va_gguf* g, const char* key, uint32_t* out, int64_t cap, int64_t* count) {
  return arr_words(g, key, false, VA_META_ARR_U32, out, cap, count);
}

int va_gguf_meta_arr_i32(const va_gguf* g, const char* key, int32_t* out, int64_t cap, int64_t* count) {
  return arr_words(g, key, true, VA_META_ARR_I32, out, cap, count);
}

int va_gguf_meta_arr_f32(const va_gguf* g, const char* key, float* out, int64_t cap, int64_t* count) {
  return arr_words(g, key, false, VA_META_ARR_F32, out, cap, count);
}

int va_gguf_meta_arr_str(const va_gguf* g, const char* key, int64_t i, const char** s, int64_t* len,
                         int64_t* count) {
  VA_META_GET(key)
  if (m->kind != VA_META_ARR_STR) return wrong_kind(key);
  const int64_t n = static_cast<int64_t>(m->strs.size());
  if (count) *count = n;
  if (s || len) {
    if (i < 0 || i >= n) return gerr(VA_ERR_INVALID, "array index out of range");
    if (s) *s = m->strs[static_cast<size_t>(i)].c_str();
    if (len) *len = static_cast<int64_t>(m->strs[static_cast<size_t>(i)].size());
  }
  return VA_OK;
}

int va_gguf_tensor_count(const va_gguf* g, int64_t* n) {
  if (!g || !n) return gerr(VA_ERR_INVALID, "null argument");
  *n = static_cast<int64_t>(g->tensors.size());
  return VA_OK;
}

int va_gguf_tensor_name(const va_gguf* g, int64_t i, const char** name, int64_t* name_len) {
  if (!g || !name || i < 0 || i >= static_cast<int64_t>(g->tensors.size()))
    return gerr(VA_ERR_INVALID, "tensor index out of range");
  const std::string& n = g->tensors[static_cast<size_t>(i)].name;
  *name = n.c_str();
  if (name_len) *name_len = static_cast<int64_t>(n.size());
  return VA_OK;
}

int va_gguf_tensor_info(const va_gguf* g, const char* name, int* dtype, int* ndims, int64_t* shape,
                        int shape_cap, uint64_t* offset) {
  if (!g || !name) return gerr(VA_ERR_INVALID, "null argument");
  const TensorInfo* t = find_tensor(g, name);
  if (!t) return gerr(VA_ERR_NOT_FOUND, std::string("tensor not found: ") + name);
  const int nd = static_cast<int>(t->dims.size());
  if (dtype) *dtype = static_cast<int>(t->dtype);
  if (ndims) *ndims = nd;
  if (offset) *offset = t->offset;
  if (shape)
    for (int i = 0; i < nd && i < shape_cap; ++i) shape[i] = static_cast<int64_t>(t->dims[nd - 1 - i]);
  if (shape && shape_cap < nd) return gerr(VA_ERR_CAPACITY, "shape buffer shorter than the tensor's rank");
  return VA_OK;
}

int va_gguf_tensor_check(const va_gguf* g, const char* name, int64_t* numel, const void** data, int64_t* nbytes) {
  va::GgufTensorRef t;
  int rc = va::gguf_tensor_ref(g, name, &t);
  if (rc) return rc;
  if (numel) *numel = t.numel;
  if (data) *data = t.data;
  if (nbytes) *nbytes = static_cast<int64_t>(t.bytes);
  return VA_OK;
}

static int convert_on_device(const va_gguf* g, const char* name, int transpose2d, float* out_dev, float* out_host,
                             int64_t cap, cudaStream_t st) {
  va::GgufTensorRef t;
  int rc = va::gguf_tensor_ref(g, name, &t);
  if (rc) return rc;
  if (!out_dev && !out_host) return gerr(VA_ERR_INVALID, "null output");
  if (out_host && t.numel > cap)
    return gerr(VA_ERR_CAPACITY, std::string("tensor '") + name + "' has " + std::to_string(t.numel) +
                                     " values, the buffer " + std::to_string(cap));
  if (t.numel == 0) return VA_OK;
  const bool tr = transpose2d && t.ndims == 2;
  const int64_t rows = tr ? t.shape[0] : 1, cols = tr ? t.shape[1] : t.numel;
  uint8_t* raw = nullptr;
  float* dev = out_dev;
  cudaError_t e = cudaMalloc(reinterpret_cast<void**>(&raw), t.bytes);
  if (e == cudaSuccess && !dev) e = cudaMalloc(reinterpret_cast<void**>(&dev), t.numel * sizeof(float));
  if (e == cudaSuccess) e = cudaMemcpyAsync(raw, t.data, t.bytes, cudaMemcpyHostToDevice, st);
  if (e == cudaSuccess) e = va::launch_gguf_convert(raw, t.dtype, rows, cols, tr ? rows : cols, tr, false, dev, st);
  if (e == cudaSuccess && out_host)
    e = cudaMemcpyAsync(out_host, dev, t.numel * sizeof(float), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (raw) cudaFree(raw);
  if (dev && dev != out_dev) cudaFree(dev);
  if (e != cudaSuccess) return gerr(VA_ERR_CUDA, std::string("gguf conversion: ") + cudaGetErrorString(e));
  return VA_OK;
}

int va_gguf_tensor_device(const va_gguf* g, const char* name, int transpose2d, float* out, void* stream) {
  if (!out) return gerr(VA_ERR_INVALID, "null output");
  return convert_on_device(g, name, transpose2d, out, nullptr, 0, static_cast<cudaStream_t>(stream));
}

int va_gguf_tensor_f32(const va_gguf* g, const char* name, int transpose2d, float* out, int64_t cap) {
  if (!out) return gerr(VA_ERR_INVALID, "null output");
  return convert_on_device(g, name, transpose2d, nullptr, out, cap, nullptr);
}

// ModelConfig::from_gguf (config.rs:219-264): required keys in the struct's order.
int va_gguf_model_config(const va_gguf* g, va_model_config* cfg) {
  if (!g || !cfg) return gerr(VA_ERR_INVALID, "null argument");
  std::memset(cfg, 0, sizeof(*cfg));
  const char* arch = nullptr;
  int64_t len = 0;
  if (va_gguf_meta_str(g, "depthanything3.arch", &arch, &len) != VA_OK || std::strcmp(arch, "depthanything3") != 0)
    return gerr(VA_ERR_INVALID, std::string("unsupported model architecture: expected 'depthanything3', found ") +
                                    (arch ? std::string("Some(\"") + arch + "\")" : std::string("None")));
  std::snprintf(cfg->arch, sizeof(cfg->arch), "%s", arch);
  auto missing = [](const char* key) {
    return gerr(VA_ERR_NOT_FOUND, std::string("missing required gguf metadata key: ") + key);
  };
  auto req_u32 = [&](const char* key, uint32_t* v) { return va_gguf_meta_u32(g, key, v) ? missing(key) : VA_OK; };
  auto req_i32 = [&](const char* key, int32_t* v) { return va_gguf_meta_i32(g, key, v) ? missing(key) : VA_OK; };
  auto req_f32 = [&](const char* key, float* v) { return va_gguf_meta_f32(g, key, v) ? missing(key) : VA_OK; };
  auto req_str = [&](const char* key, char* dst, size_t cap) {
    const char* s;
    int64_t n;
    if (va_gguf_meta_str(g, key, &s, &n)) return missing(key);
    if (static_cast<size_t>(n) >= cap) return gerr(VA_ERR_CAPACITY, std::string("string too long for ") + key);
    std::memcpy(dst, s, static_cast<size_t>(n) + 1);
    return VA_OK;
  };
  auto req_vec3 = [&](const char* key, float* dst) {
    int64_t n = 0;
    if (va_gguf_meta_arr_f32(g, key, nullptr, 0, &n)) return missing(key);
    if (n != 3)
      return gerr(VA_ERR_FORMAT, std::string("malformed gguf metadata for key ") + key + ": expected 3 elements, got " +
                                     std::to_string(n));
    return va_gguf_meta_arr_f32(g, key, dst, 3, &n);
  };
  int rc;
  if ((rc = req_u32("depthanything3.patch_size", &cfg->patch_size))) return rc;
  if (va_gguf_meta_u32(g, "depthanything3.img.resize_target", &cfg->image_size) &&
      va_gguf_meta_u32(g, "depthanything3.image_size", &cfg->image_size))
    return missing("depthanything3.img.resize_target");
  if ((rc = req_u32("depthanything3.vit.embed_dim", &cfg->embed_dim))) return rc;
  if ((rc = req_u32("depthanything3.vit.depth", &cfg->depth))) return rc;
  if ((rc = req_u32("depthanything3.vit.num_heads", &cfg->num_heads))) return rc;
  if ((rc = req_u32("depthanything3.vit.head_dim", &cfg->head_dim))) return rc;
  if ((rc = req_u32("depthanything3.vit.mlp_hidden", &cfg->mlp_hidden))) return rc;
  if ((rc = req_u32("depthanything3.vit.num_register_tokens", &cfg->num_register))) return rc;
  if ((rc = req_i32("depthanything3.vit.rope_start", &cfg->rope_start))) return rc;
  if ((rc = req_i32("depthanything3.vit.qknorm_start", &cfg->qknorm_start))) return rc;
  if ((rc = req_f32("depthanything3.vit.rope_freq", &cfg->rope_freq))) return rc;
  if ((rc = req_f32("depthanything3.vit.ln_eps", &cfg->ln_eps))) return rc;
  {
    int64_t n = 0;
    const char* key = "depthanything3.vit.out_layers";
    if (va_gguf_meta_arr_i32(g, key, nullptr, 0, &n)) return missing(key);
    if (n > VA_MAX_OUT_LAYERS) return gerr(VA_ERR_CAPACITY, "more out_layers than VA_MAX_OUT_LAYERS");
    va_gguf_meta_arr_i32(g, key, cfg->out_layers, VA_MAX_OUT_LAYERS, &n);
    cfg->n_out_layers = static_cast<int32_t>(n);
  }
  {
    const char* s;
    int64_t n;
    if (va_gguf_meta_str(g, "depthanything3.vit.ffn_type", &s, &n) == VA_OK) {
      if (static_cast<size_t>(n) >= sizeof(cfg->ffn_type)) return gerr(VA_ERR_CAPACITY, "ffn_type too long");
      std::memcpy(cfg->ffn_type, s, static_cast<size_t>(n) + 1);
    } else {
      std::snprintf(cfg->ffn_type, sizeof(cfg->ffn_type), "mlp");
    }
  }
  if (va_gguf_meta_i32(g, "depthanything3.vit.alt_start", &cfg->alt_start)) cfg->alt_start = -1;
  int b = 1;
  cfg->cat_token = va_gguf_meta_bool(g, "depthanything3.vit.cat_token", &b) ? 1 : b;
  if ((rc = req_u32("depthanything3.head.features", &cfg->head_features))) return rc;
  if (va_gguf_meta_f32(g, "depthanything3.head.max_depth", &cfg->head_max_depth)) cfg->head_max_depth = 0.f;
  b = 1;
  cfg->head_pos_embed = va_gguf_meta_bool(g, "depthanything3.head.pos_embed", &b) ? 1 : b;
  if ((rc = req_vec3("depthanything3.img.mean", cfg->img_mean))) return rc;
  if ((rc = req_vec3("depthanything3.img.std", cfg->img_std))) return rc;
  if ((rc = req_str("depthanything3.img.resize_mode", cfg->img_resize_mode, sizeof(cfg->img_resize_mode)))) return rc;
  if ((rc = req_u32("depthanything3.cam.dim_in", &cfg->cam_dim_in))) return rc;
  return VA_OK;
}

}  // extern "C"
