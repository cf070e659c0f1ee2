// Blob producer: an HF Qwen3 safetensors checkpoint -> the pqwf blob on the
// device (tools/convert_pqwf.py:125-219 + tools/pqwf.py:42-89, 279-360).
//
// The file is read in row chunks into pinned memory and copied to the device,
// where every weight matrix is quantised per output row exactly as
// pqwf.quantize_into does it: widen BF16 / F16 / F32 to float32,
// scale = absmax * (1/127), q = rne(x / scale) saturated to +-127 (NaN -> 0),
// int8 rows at the matrix offset, float32 scales right after them.  Norm
// weights are widened on the host; the RoPE tables are computed on the host in
// double precision as convert_pqwf.rope_tables does.  Layers and vocabulary
// rows beyond the layout are not read (the converter's --layers / --vocab).
//
// F16 tensors: pqwf.SafeTensors views them as uint16 and widens the bit
// patterns as unsigned integers (pqwf.py:302, 313, 320).  By default they are
// decoded as IEEE half here; Q3_CONVERT_F16_AS_UINT16 reproduces the
// reference's reading bit for bit.
#include <stdio.h>
#include <string.h>

#include <cmath>
#include <map>
#include <string>
#include <vector>

#include <cuda_fp16.h>

#include "q3_common.cuh"
#include "q3_json.h"

namespace {

struct Tensor {
  int dtype = -1;                 // 0 F32, 1 BF16, 2 F16
  std::vector<uint64_t> shape;
  uint64_t begin = 0, end = 0;    // absolute file offsets
};

struct SafeTensors {
  FILE *f = nullptr;
  std::map<std::string, Tensor> t;
  ~SafeTensors() { if (f) fclose(f); }
  int open(const char *path) {
    f = fopen(path, "rb");
    if (!f) return Q3_ERR_NULL;
    uint64_t hlen = 0;
    if (fread(&hlen, 8, 1, f) != 1 || hlen == 0 || hlen > (1ull << 30)) return Q3_ERR_SHAPE;
    std::string h(hlen, '\0');
    if (fread(&h[0], 1, hlen, f) != hlen) return Q3_ERR_SHAPE;
    if (fseeko(f, 0, SEEK_END)) return Q3_ERR_SHAPE;
    const uint64_t fsize = static_cast<uint64_t>(ftello(f));
    q3json::Parser jp{h.data(), h.data() + h.size()};
    q3json::Value root = jp.value();
    if (!jp.ok || root.kind != q3json::Value::OBJ) return Q3_ERR_SHAPE;
    for (const auto &kv : root.obj) {
      if (kv.first == "__metadata__") continue;
      const q3json::Value *dt = kv.second.get("dtype"), *sh = kv.second.get("shape"),
                 *of = kv.second.get("data_offsets");
      if (!dt || !sh || !of || dt->kind != q3json::Value::STR || sh->kind != q3json::Value::ARR ||
          of->kind != q3json::Value::ARR || of->arr.size() != 2)
        return Q3_ERR_SHAPE;
      // every size is a non-negative integer (no wrap-around into the header)
      auto count = [](const q3json::Value &v, uint64_t &out) {
        if (v.kind != q3json::Value::NUM || !(v.num >= 0.0) || v.num > 9007199254740992.0 ||
            v.num != static_cast<double>(static_cast<uint64_t>(v.num)))
          return false;
        out = static_cast<uint64_t>(v.num);
        return true;
      };
      Tensor x;
      x.dtype = dt->str == "F32" ? 0 : dt->str == "BF16" ? 1 : dt->str == "F16" ? 2 : -1;
      for (const q3json::Value &d : sh->arr) {
        uint64_t v;
        if (!count(d, v) || v > (1ull << 40)) return Q3_ERR_SHAPE;
        x.shape.push_back(v);
      }
      uint64_t a, b;
      if (!count(of->arr[0], a) || !count(of->arr[1], b)) return Q3_ERR_SHAPE;
      x.begin = 8 + hlen + a;
      x.end = 8 + hlen + b;
      uint64_t n = x.dtype < 0 ? 0 : (x.dtype == 0 ? 4 : 2);
      for (uint64_t d : x.shape) {
        if (d && n > UINT64_MAX / d) return Q3_ERR_SHAPE;
        n *= d;
      }
      if (x.end < x.begin || x.end > fsize || (x.dtype >= 0 && x.end - x.begin != n))
        return Q3_ERR_SHAPE;
      t[kv.first] = x;
    }
    return Q3_OK;
  }
  const Tensor *find(const std::string &name) const {
    auto it = t.find(name);
    return it == t.end() ? nullptr : &it->second;
  }
};

// dtype codes: 0 F32, 1 BF16, 2 F16, 3 F16 read as uint16 (reference mode)
int esize(int dtype) { return dtype == 0 ? 4 : 2; }

float widen(const unsigned char *p, int dtype) {
  if (dtype == 0) { float v; memcpy(&v, p, 4); return v; }
  uint16_t b;
  memcpy(&b, p, 2);
  if (dtype == 1) { const uint32_t u = static_cast<uint32_t>(b) << 16; float v; memcpy(&v, &u, 4); return v; }
  if (dtype == 3) return static_cast<float>(b);
  // IEEE half -> float (exact)
  const uint32_t s = (b >> 15) & 1u, e = (b >> 10) & 31u, m = b & 1023u;
  float v;
  if (e == 0) v = std::ldexp(static_cast<float>(m), -24);
  else if (e == 31) v = m ? NAN : INFINITY;
  else v = std::ldexp(static_cast<float>(m | 1024u), static_cast<int>(e) - 25);
  return s ? -v : v;
}

// ------------------------------------------------------------ device quantiser
__device__ __forceinline__ float dev_widen(const unsigned char *row, int dtype, int c) {
  if (dtype == 0) return reinterpret_cast<const float *>(row)[c];
  const uint16_t b = reinterpret_cast<const uint16_t *>(row)[c];
  if (dtype == 1) return __uint_as_float(static_cast<uint32_t>(b) << 16);
  if (dtype == 3) return static_cast<float>(b);
  return __half2float(__ushort_as_half(b));
}

// one CTA per row: pqwf.quantize_rows
__global__ void __launch_bounds__(256) k_quant_rows_dt(const unsigned char *src, int dtype, int cols,
                                                       int8_t *q, float *scale) {
  const int r = blockIdx.x, t = threadIdx.x;
  const unsigned char *row = src + static_cast<size_t>(r) * cols * (dtype == 0 ? 4 : 2);
  __shared__ float red[8];
  float mx = 0.0f;
  int nan = 0;
  for (int c = t; c < cols; c += 256) {
    const float v = dev_widen(row, dtype, c);
    nan |= v != v;
    mx = fmaxf(mx, fabsf(v));
  }
  mx = q3::warp_tree_max(mx);
  if ((t & 31) == 0) red[t >> 5] = mx;
  // np.max propagates NaN: such a row gets a NaN scale and all-zero codes
  nan = __syncthreads_or(nan);
  mx = 0.0f;
#pragma unroll
  for (int w = 0; w < 8; ++w) mx = fmaxf(mx, red[w]);
  const float s = nan ? __int_as_float(0x7FC00000) : __fmul_rn(mx, q3::kInv127);
  for (int c = t; c < cols; c += 256)
    q[static_cast<size_t>(r) * cols + c] = static_cast<int8_t>(q3::quant1(dev_widen(row, dtype, c), s));
  if (t == 0) scale[r] = s;
}

struct Ctx {
  SafeTensors st;
  char *blob;
  cudaStream_t s;
  unsigned char *pinned = nullptr;
  unsigned char *dstage = nullptr;
  size_t cap = 0;
  bool f16_bits = false;
  int dt(const Tensor *x) const { return x->dtype == 2 && f16_bits ? 3 : x->dtype; }
  ~Ctx() {
    if (pinned) cudaFreeHost(pinned);
    if (dstage) cudaFree(dstage);
  }
};

int cuda_err(cudaError_t e) {
  if (e == cudaSuccess) return Q3_OK;
  q3h::set_cuda_error(e);
  return Q3_ERR_CUDA;
}

// rows [0, rows) of a 2-D tensor, quantised into the blob
int quantize_into(Ctx &c, const std::string &name, int64_t q_off, int64_t s_off, uint64_t rows,
                  uint64_t cols) {
  const Tensor *x = c.st.find(name);
  if (!x || x->dtype < 0 || x->shape.size() != 2 || x->shape[1] != cols || x->shape[0] < rows)
    return Q3_ERR_SHAPE;
  const size_t row_bytes = cols * esize(x->dtype);
  const uint64_t chunk = std::max<uint64_t>(1, c.cap / row_bytes);
  for (uint64_t r0 = 0; r0 < rows; r0 += chunk) {
    const uint64_t n = std::min(chunk, rows - r0);
    // the previous chunk's copy must have left the pinned buffer
    Q3_TRY(cuda_err(cudaStreamSynchronize(c.s)));
    if (fseeko(c.st.f, static_cast<off_t>(x->begin + r0 * row_bytes), SEEK_SET) ||
        fread(c.pinned, 1, n * row_bytes, c.st.f) != n * row_bytes)
      return Q3_ERR_SHAPE;
    Q3_TRY(cuda_err(cudaMemcpyAsync(c.dstage, c.pinned, n * row_bytes, cudaMemcpyHostToDevice, c.s)));
    k_quant_rows_dt<<<static_cast<unsigned>(n), 256, 0, c.s>>>(
        c.dstage, c.dt(x), static_cast<int>(cols),
        reinterpret_cast<int8_t *>(c.blob + q_off + r0 * cols),
        reinterpret_cast<float *>(c.blob + s_off + r0 * 4));
    Q3_TRY(q3h::launch_status());
  }
  return Q3_OK;
}

int put_vector(Ctx &c, const std::string &name, int64_t off, uint64_t n) {
  const Tensor *x = c.st.find(name);
  if (!x || x->dtype < 0 || x->shape.size() != 1 || x->shape[0] != n) return Q3_ERR_SHAPE;
  std::vector<unsigned char> raw(n * esize(x->dtype));
  if (fseeko(c.st.f, static_cast<off_t>(x->begin), SEEK_SET) || fread(raw.data(), 1, raw.size(), c.st.f) != raw.size())
    return Q3_ERR_SHAPE;
  std::vector<float> v(n);
  for (uint64_t i = 0; i < n; ++i) v[i] = widen(raw.data() + i * esize(x->dtype), c.dt(x));
  Q3_TRY(cuda_err(cudaMemcpyAsync(c.blob + off, v.data(), 4 * n, cudaMemcpyHostToDevice, c.s)));
  return cuda_err(cudaStreamSynchronize(c.s));   // v is pageable and goes out of scope
}

}  // namespace

extern "C" int q3_safetensors_tensor(const char *path, const char *name, int32_t *dtype,
                                     uint64_t *shape, int32_t *ndim) {
  if (!path || !name || !dtype || !shape || !ndim) return Q3_ERR_NULL;
  SafeTensors st;
  Q3_TRY(st.open(path));
  const Tensor *x = st.find(name);
  if (!x) return Q3_ERR_SHAPE;
  *dtype = x->dtype;
  *ndim = static_cast<int32_t>(x->shape.size());
  for (size_t i = 0; i < x->shape.size() && i < 4; ++i) shape[i] = x->shape[i];
  return Q3_OK;
}

extern "C" int q3_blob_from_safetensors(const char *path, const q3_layout *layout, double rope_theta,
                                        uint32_t flags, void *blob, void *stream) {
  if (!path || !layout || !blob) return Q3_ERR_NULL;
  if (flags & ~static_cast<uint32_t>(Q3_CONVERT_F16_AS_UINT16)) return Q3_ERR_MODE;
  const q3_layout &L = *layout;
  const int64_t *o = L.off;
  Ctx c;
  Q3_TRY(c.st.open(path));
  c.blob = static_cast<char *>(blob);
  c.s = static_cast<cudaStream_t>(stream);
  c.cap = 64u << 20;
  c.f16_bits = flags & Q3_CONVERT_F16_AS_UINT16;
  Q3_TRY(cuda_err(cudaMallocHost(&c.pinned, c.cap)));
  Q3_TRY(cuda_err(cudaMalloc(&c.dstage, c.cap)));
  const uint64_t H = L.hidden, V = L.vocab, I = L.inter, HD = L.head_dim;
  const uint64_t QW = L.heads * HD, KW = L.kv_heads * HD, MS = L.max_seq, HALF = HD / 2;

  Q3_TRY(put_vector(c, "model.norm.weight", o[Q3_OFF_NF], H));
  {   // convert_pqwf.rope_tables: float64 angles pos * theta^(-i/half)
    std::vector<float> cs(MS * HALF), sn(MS * HALF);
    for (uint64_t i = 0; i < HALF; ++i) {
      const double inv = 1.0 / std::pow(rope_theta, static_cast<double>(i) / static_cast<double>(HALF));
      for (uint64_t p = 0; p < MS; ++p) {
        const double a = static_cast<double>(p) * inv;
        cs[p * HALF + i] = static_cast<float>(std::cos(a));
        sn[p * HALF + i] = static_cast<float>(std::sin(a));
      }
    }
    Q3_TRY(cuda_err(cudaMemcpyAsync(c.blob + o[Q3_OFF_COS], cs.data(), 4 * cs.size(), cudaMemcpyHostToDevice, c.s)));
    Q3_TRY(cuda_err(cudaMemcpyAsync(c.blob + o[Q3_OFF_SIN], sn.data(), 4 * sn.size(), cudaMemcpyHostToDevice, c.s)));
    Q3_TRY(cuda_err(cudaStreamSynchronize(c.s)));
  }
  Q3_TRY(quantize_into(c, "model.embed_tokens.weight", o[Q3_OFF_EMB], o[Q3_OFF_EMB] + V * H, V, H));
  const std::string lm = c.st.find("lm_head.weight") ? "lm_head.weight" : "model.embed_tokens.weight";
  Q3_TRY(quantize_into(c, lm, o[Q3_OFF_LM], o[Q3_OFF_LM] + V * H, V, H));
  struct P { const char *name; int data, scale; uint64_t rows, cols; };
  const P projs[7] = {{"self_attn.q_proj", Q3_OFF_LQ, Q3_OFF_LQ_SCALE, QW, H},
                      {"self_attn.k_proj", Q3_OFF_LK, Q3_OFF_LK_SCALE, KW, H},
                      {"self_attn.v_proj", Q3_OFF_LV, Q3_OFF_LV_SCALE, KW, H},
                      {"self_attn.o_proj", Q3_OFF_LO, Q3_OFF_LO_SCALE, H, QW},
                      {"mlp.gate_proj", Q3_OFF_LG, Q3_OFF_LG_SCALE, I, H},
                      {"mlp.up_proj", Q3_OFF_LU, Q3_OFF_LU_SCALE, I, H},
                      {"mlp.down_proj", Q3_OFF_LD, Q3_OFF_LD_SCALE, H, I}};
  for (uint32_t li = 0; li < L.layers; ++li) {
    const std::string pre = "model.layers." + std::to_string(li) + ".";
    const int64_t base = o[Q3_OFF_LQ] + static_cast<int64_t>(li) * o[Q3_OFF_LAYERW_STRIDE];
    for (const P &p : projs)
      Q3_TRY(quantize_into(c, pre + p.name + ".weight", base + (o[p.data] - o[Q3_OFF_LQ]),
                           base + (o[p.scale] - o[Q3_OFF_LQ]), p.rows, p.cols));
    const int64_t nb = o[Q3_OFF_N1] + static_cast<int64_t>(li) * o[Q3_OFF_LAYERN_STRIDE];
    Q3_TRY(put_vector(c, pre + "input_layernorm.weight", nb, H));
    Q3_TRY(put_vector(c, pre + "self_attn.q_norm.weight", nb + (o[Q3_OFF_NQ] - o[Q3_OFF_N1]), HD));
    Q3_TRY(put_vector(c, pre + "self_attn.k_norm.weight", nb + (o[Q3_OFF_NK] - o[Q3_OFF_N1]), HD));
    Q3_TRY(put_vector(c, pre + "post_attention_layernorm.weight", nb + (o[Q3_OFF_N2] - o[Q3_OFF_N1]), H));
  }
  return cuda_err(cudaStreamSynchronize(c.s));
}
