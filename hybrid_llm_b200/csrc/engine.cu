// Native serving engine behind the reference engine's C API
// (llmy_cuda/include/llmy.h:27-88; llmy_cuda/src/llmy.cpp:21-210 and
// model.cpp:1774-1972): a `.llmy` checkpoint mapped and uploaded by C++ code,
// each token one cooperative launch of the persistent decode step
// (decode_persistent.cu).  No Python on this path.
//
// Loading (llmy_load) follows the file layout of llmy_cuda/include/checkpoint.h
// (written by llmy_cuda/tools/convert_checkpoint.py): "LLMY", u32 version 1,
// u32 config length, `key=value` configuration lines, u32 tensor count, one
// 108-byte index entry per tensor (u32 name length, char name[64], u32 dtype
// 0 f32 / 1 f16 / 2 bf16, u32 ndim, u32 shape[4], u64 offset, u64 bytes), and
// the payloads from the first 4096-byte boundary after the index.  Missing
// configuration keys take the reference engine's defaults
// (llmy_cuda/include/config.h).
//
// The device weights are the ones the persistent step reads:
//   embed [V, D] bf16 (tied LM head), stream_seed [D] f32, collapse [D, D]
//   bf16, final_norm [D] f32;
//   per block: mixer_norm / ffn_norm [D] f32; router_fold [E, D] f32 =
//   router.logits * ffn_norm * router.norm (the two RMSNorms before the router
//   reduce to per-token scales); w13 [E, 2F, D] (gate / up interleaved by
//   llmyb_moe_pack_w13), w2 [E, D, F] bf16;
//   CSA: w_in [2 H Dh + D, D] bf16 = query | key | W_o value, where W_o =
//   bf16(out . local_out) and the value rows are bf16(W_o . value) formed in
//   fp32 on the device (the attention output is then the block output, the
//   ring caching W_o W_v x);
//   GDN: w_in = q | k | v | gate | beta rows (zero rows to a multiple of 8),
//   beta bias, decay logits, out_proj, conv [D, 4] f32.
// A state holds, per loop and block, the CSA key ring [W, H Dh] and folded
// value ring [W, D] bf16, or the GDN state [H, 64, 64] f32 and conv history
// [3, D] bf16, plus the step's scratch.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "common.cuh"
#include "../../include/llmyb.h"
#include "../../include/llmy.h"

namespace {

// ------------------------------------------------------------ checkpoint file
struct FileTensor {
  int dtype = 0;                 // 0 f32, 1 f16, 2 bf16
  std::vector<int64_t> shape;
  const uint8_t* data = nullptr;
  uint64_t nbytes = 0;
  int64_t numel() const {
    int64_t n = 1;
    for (int64_t s : shape) n *= s;
    return n;
  }
};

class LlmyFile {
 public:
  explicit LlmyFile(const std::string& path) {
    fd_ = ::open(path.c_str(), O_RDONLY);
    if (fd_ < 0) throw std::runtime_error("cannot open " + path);
    struct stat st;
    if (fstat(fd_, &st) != 0) throw std::runtime_error("cannot stat " + path);
    size_ = static_cast<size_t>(st.st_size);
    if (size_ < 16) throw std::runtime_error(path + ": not an .llmy file");
    void* m = mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd_, 0);
    if (m == MAP_FAILED) throw std::runtime_error("cannot map " + path);
    base_ = static_cast<const uint8_t*>(m);
    if (std::memcmp(base_, "LLMY", 4) != 0) throw std::runtime_error(path + ": not an .llmy file");
    const uint32_t version = u32(4), cfg_len = u32(8);
    if (version != 1) throw std::runtime_error(path + ": unsupported version " + std::to_string(version));
    if (12ull + cfg_len + 4 > size_) throw std::runtime_error(path + ": truncated configuration");
    parse_config(std::string(reinterpret_cast<const char*>(base_ + 12), cfg_len));
    uint64_t pos = 12ull + cfg_len;
    const uint32_t n = u32(pos);
    pos += 4;
    const uint64_t index_end = pos + 108ull * n;
    if (index_end > size_) throw std::runtime_error(path + ": index runs past the end of the file");
    const uint64_t data_start = (index_end + 4095) / 4096 * 4096;
    for (uint32_t i = 0; i < n; ++i, pos += 108) {
      const uint32_t name_len = u32(pos), dtype = u32(pos + 68), ndim = u32(pos + 72);
      if (name_len > 63 || dtype > 2 || ndim > 4)
        throw std::runtime_error(path + ": bad index entry " + std::to_string(i));
      FileTensor t;
      t.dtype = static_cast<int>(dtype);
      for (uint32_t d = 0; d < ndim; ++d) t.shape.push_back(u32(pos + 76 + 4 * d));
      const uint64_t off = u64(pos + 92);
      t.nbytes = u64(pos + 100);
      if (data_start + off + t.nbytes > size_)
        throw std::runtime_error(path + ": tensor " + std::to_string(i) + " runs past the end");
      const int64_t esize = dtype == 0 ? 4 : 2;
      if (static_cast<uint64_t>(t.numel() * esize) != t.nbytes)
        throw std::runtime_error(path + ": tensor " + std::to_string(i) + " size mismatch");
      t.data = base_ + data_start + off;
      tensors_[std::string(reinterpret_cast<const char*>(base_ + pos + 4), name_len)] = t;
    }
  }
  ~LlmyFile() {
    if (base_) munmap(const_cast<uint8_t*>(base_), size_);
    if (fd_ >= 0) ::close(fd_);
  }
  LlmyFile(const LlmyFile&) = delete;
  LlmyFile& operator=(const LlmyFile&) = delete;

  const FileTensor& tensor(const std::string& name) const {
    auto it = tensors_.find(name);
    if (it == tensors_.end()) throw std::runtime_error("missing tensor " + name);
    return it->second;
  }
  bool has(const std::string& name) const { return tensors_.count(name) != 0; }
  bool has_key(const std::string& k) const { return config_.count(k) != 0; }
  const std::string& value(const std::string& k) const { return config_.at(k); }

 private:
  uint32_t u32(uint64_t off) const {
    uint32_t v;
    std::memcpy(&v, base_ + off, 4);
    return v;
  }
  uint64_t u64(uint64_t off) const {
    uint64_t v;
    std::memcpy(&v, base_ + off, 8);
    return v;
  }
  void parse_config(const std::string& text) {
    size_t start = 0;
    while (start < text.size()) {
      size_t end = text.find('\n', start);
      if (end == std::string::npos) end = text.size();
      std::string line = text.substr(start, end - start);
      start = end + 1;
      while (!line.empty() && (line.back() == '\r' || line.back() == ' ')) line.pop_back();
      if (line.empty() || line[0] == '#') continue;
      const size_t eq = line.find('=');
      if (eq == std::string::npos) continue;
      config_[line.substr(0, eq)] = line.substr(eq + 1);
    }
  }

  int fd_ = -1;
  size_t size_ = 0;
  const uint8_t* base_ = nullptr;
  std::map<std::string, std::string> config_;
  std::map<std::string, FileTensor> tensors_;
};

int32_t cfg_int(const LlmyFile& f, const char* key, int32_t dflt) {
  if (!f.has_key(key)) return dflt;
  const std::string& v = f.value(key);
  char* end = nullptr;
  const long x = std::strtol(v.c_str(), &end, 10);
  if (end == v.c_str() || *end != '\0')
    throw std::runtime_error(std::string("configuration ") + key + ": expected an integer, got " + v);
  return static_cast<int32_t>(x);
}

bool cfg_bool(const LlmyFile& f, const char* key, bool dflt) {
  if (!f.has_key(key)) return dflt;
  const std::string& v = f.value(key);
  if (v == "1" || v == "true" || v == "True" || v == "yes") return true;
  if (v == "0" || v == "false" || v == "False" || v == "no") return false;
  throw std::runtime_error(std::string("configuration ") + key + ": expected a boolean, got " + v);
}

// ---------------------------------------------------------- host conversions
float half_to_float(uint16_t h) {  // IEEE 754 binary16 -> binary32
  const int sign = h >> 15, ex = (h >> 10) & 0x1f, man = h & 0x3ff;
  float v;
  if (ex == 0) v = std::ldexp(static_cast<float>(man), -24);
  else if (ex == 31) v = man ? NAN : INFINITY;
  else v = std::ldexp(static_cast<float>(man | 0x400), ex - 25);
  return sign ? -v : v;
}

uint16_t float_to_bf16(float f) {  // round to nearest even
  uint32_t u;
  std::memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return static_cast<uint16_t>((u >> 16) | 0x40);
  u += 0x7fffu + ((u >> 16) & 1u);
  return static_cast<uint16_t>(u >> 16);
}

std::vector<float> as_f32(const FileTensor& t) {
  const int64_t n = t.numel();
  std::vector<float> out(static_cast<size_t>(n));
  if (t.dtype == 0) {
    std::memcpy(out.data(), t.data, static_cast<size_t>(n) * 4);
  } else {
    for (int64_t i = 0; i < n; ++i) {
      uint16_t h;
      std::memcpy(&h, t.data + 2 * i, 2);
      if (t.dtype == 1) {
        out[i] = half_to_float(h);
      } else {
        const uint32_t u = static_cast<uint32_t>(h) << 16;
        std::memcpy(&out[i], &u, 4);
      }
    }
  }
  return out;
}

std::vector<uint16_t> as_bf16(const FileTensor& t) {
  const int64_t n = t.numel();
  std::vector<uint16_t> out(static_cast<size_t>(n));
  if (t.dtype == 2) {
    std::memcpy(out.data(), t.data, static_cast<size_t>(n) * 2);
  } else {
    const std::vector<float> f = as_f32(t);
    for (int64_t i = 0; i < n; ++i) out[i] = float_to_bf16(f[i]);
  }
  return out;
}

std::string shape_str(const std::vector<int64_t>& s) {
  std::string r = "[";
  for (size_t i = 0; i < s.size(); ++i) r += (i ? ", " : "") + std::to_string(s[i]);
  return r + "]";
}

void check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

void check_status(int32_t st, const char* what) {
  if (st != 0) throw std::runtime_error(std::string(what) + " failed with status " + std::to_string(st));
}

// ------------------------------------------------------------- load kernels
// c[M, N] = a[M, K] . b[K, N], fp32 (the CSA value-row fold; load time only)
__global__ void fold_matmul_kernel(const float* __restrict__ a, const float* __restrict__ b,
                                   float* __restrict__ c, int M, int K, int N) {
  __shared__ float ta[16][17], tb[16][17];
  const int ty = threadIdx.y, tx = threadIdx.x;
  const int row = blockIdx.y * 16 + ty, col = blockIdx.x * 16 + tx;
  float acc = 0.f;
  for (int k0 = 0; k0 < K; k0 += 16) {
    ta[ty][tx] = (row < M && k0 + tx < K) ? a[static_cast<int64_t>(row) * K + k0 + tx] : 0.f;
    tb[ty][tx] = (k0 + ty < K && col < N) ? b[static_cast<int64_t>(k0 + ty) * N + col] : 0.f;
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < 16; ++kk) acc = fmaf(ta[ty][kk], tb[kk][tx], acc);
    __syncthreads();
  }
  if (row < M && col < N) c[static_cast<int64_t>(row) * N + col] = acc;
}

// x <- float(bf16(x)); optionally also the bf16 copy
__global__ void round_bf16_kernel(float* __restrict__ x, __nv_bfloat16* __restrict__ out, int64_t n) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const __nv_bfloat16 h = __float2bfloat16_rn(x[i]);
    x[i] = __bfloat162float(h);
    if (out) out[i] = h;
  }
}

// ------------------------------------------------------------------- model
struct BlockDims {
  int kind = 0;   // 0 CSA, 1 GDN
  int rows = 0;
};

}  // namespace

struct llmy_model {
  int device = 0;
  int vocab = 0, d = 0, file_loops = 0, num_loops = 0, n_blocks = 0;
  int csa_heads = 0, csa_head_dim = 0, window = 0;
  int gdn_heads = 0, gdn_dim = 0;
  int n_experts = 0, top_k = 0, ffn = 0;
  int max_rows = 0, grid = 0;
  bool has_csa = false, has_gdn = false;
  std::vector<int> kinds;                   // per block: 0 CSA, 1 GDN
  std::vector<void*> allocs;                // every device buffer of the model
  llmyb_pblock* blocks = nullptr;           // device table [n_blocks]
  void* embed = nullptr;
  float* stream_seed = nullptr;
  void* collapse = nullptr;
  float* final_norm = nullptr;

  void* alloc(size_t bytes) {
    void* p = nullptr;
    check(cudaMalloc(&p, bytes ? bytes : 16), "cudaMalloc");
    allocs.push_back(p);
    return p;
  }
  template <typename T>
  T* upload(const std::vector<T>& host) {
    T* p = static_cast<T*>(alloc(host.size() * sizeof(T)));
    check(cudaMemcpy(p, host.data(), host.size() * sizeof(T), cudaMemcpyHostToDevice), "upload");
    return p;
  }
  ~llmy_model() {
    for (void* p : allocs) cudaFree(p);
  }
};

struct llmy_state {
  llmy_model* m = nullptr;
  int loops = 0;                            // loop slots held
  int last_executed_loops = 0;
  std::vector<void*> allocs;
  std::vector<std::pair<void*, size_t>> recurrent;  // zeroed by reset
  llmyb_pdecode p{};
  int64_t* io = nullptr;                    // device [2]: token, then position (int32)
  int64_t* io_host = nullptr;               // pinned [2]
  int32_t* status_host = nullptr;           // pinned [1]
  int64_t* prompt = nullptr;                // device prompt ids
  int64_t prompt_cap = 0;

  void* alloc(size_t bytes, bool zero_on_reset = false) {
    void* p = nullptr;
    check(cudaMalloc(&p, bytes ? bytes : 16), "cudaMalloc");
    allocs.push_back(p);
    check(cudaMemset(p, 0, bytes ? bytes : 16), "cudaMemset");
    if (zero_on_reset) recurrent.emplace_back(p, bytes);
    return p;
  }
  ~llmy_state() {
    for (void* p : allocs) cudaFree(p);
    if (io_host) cudaFreeHost(io_host);
    if (status_host) cudaFreeHost(status_host);
  }
};

namespace {

const FileTensor& expect(const LlmyFile& f, const std::string& name,
                         std::initializer_list<int64_t> shape) {
  const FileTensor& t = f.tensor(name);
  const std::vector<int64_t> want(shape);
  if (t.shape != want) {
    // a [1, D] / [D] difference is a layout choice of the writer, not an error
    if (t.numel() != [&] { int64_t n = 1; for (int64_t s : want) n *= s; return n; }() ||
        (t.shape.size() > 1 && want.size() > 1))
      throw std::runtime_error(name + " has shape " + shape_str(t.shape) + ", expected " +
                               shape_str(want));
  }
  return t;
}

// Experts of one projection as [E, rows, cols]: the converter's stacked tensor
// (moe.experts.<name>.weight) or the per-expert ones (moe.experts.<e>.<name>.weight).
std::vector<uint16_t> expert_stack(const LlmyFile& f, const std::string& p, const char* name,
                                   int E, int rows, int cols) {
  const std::string stacked = p + "moe.experts." + name + ".weight";
  if (f.has(stacked)) return as_bf16(expect(f, stacked, {E, rows, cols}));
  std::vector<uint16_t> out;
  out.reserve(static_cast<size_t>(E) * rows * cols);
  for (int e = 0; e < E; ++e) {
    const std::vector<uint16_t> one = as_bf16(
        expect(f, p + "moe.experts." + std::to_string(e) + "." + name + ".weight", {rows, cols}));
    out.insert(out.end(), one.begin(), one.end());
  }
  return out;
}

void load_config(const LlmyFile& f, llmy_model& m) {
  auto fail = [](const std::string& why) {
    throw std::runtime_error(why + " (served by the Python engine, hybrid_llm_b200.engine)");
  };
  m.vocab = cfg_int(f, "vocab_size", 32000);
  m.d = cfg_int(f, "d_model", 768);
  m.file_loops = m.num_loops = cfg_int(f, "num_loops", 2);
  if (cfg_int(f, "stem_blocks", 2) || cfg_int(f, "tail_blocks", 2))
    fail("stem / tail dense blocks are not served by the native engine");
  if (cfg_bool(f, "mhc.enabled", true)) fail("hyper-connections (mhc.enabled) are not served natively");
  if (cfg_bool(f, "router.context_aware", true))
    fail("the router's context (router.context_aware) is not served natively");
  if (cfg_int(f, "moe.shared_experts", 4)) fail("shared experts are not served natively");
  if (cfg_bool(f, "loop_attnres.enabled", false)) fail("loop memory is not served natively");
  if (cfg_bool(f, "adaptive_loops.enabled", false)) fail("adaptive halting is not served natively");
  if (f.has_key("gdn.sensitive_state_dtype")) {
    const std::string& v = f.value("gdn.sensitive_state_dtype");
    if (v != "float32" && v != "fp32") fail("the GDN state is kept in float32 only");
  }
  if (!f.has_key("recurrent_layout")) throw std::runtime_error("configuration has no recurrent_layout");
  const std::string& layout = f.value("recurrent_layout");
  size_t start = 0;
  while (start <= layout.size()) {
    size_t end = layout.find(',', start);
    if (end == std::string::npos) end = layout.size();
    std::string item = layout.substr(start, end - start);
    item.erase(0, item.find_first_not_of(" '\"[]"));
    item.erase(item.find_last_not_of(" '\"[]") + 1);
    if (!item.empty()) {
      const std::string kind = item.substr(0, 3);
      if (kind == "csa") m.kinds.push_back(0);
      else if (kind == "gdn") m.kinds.push_back(1);
      else fail("recurrent block kind '" + item + "' is not served natively");
    }
    start = end + 1;
  }
  m.n_blocks = static_cast<int>(m.kinds.size());
  if (m.n_blocks == 0) throw std::runtime_error("recurrent_layout is empty");
  m.has_csa = std::count(m.kinds.begin(), m.kinds.end(), 0) > 0;
  m.has_gdn = std::count(m.kinds.begin(), m.kinds.end(), 1) > 0;
  m.csa_heads = cfg_int(f, "csa.index_heads", 8);
  m.csa_head_dim = cfg_int(f, "csa.index_head_dim", 64);
  m.window = cfg_int(f, "csa.local_window", 512);
  const int ratio = cfg_int(f, "csa.temporal_compression", 4);
  if (m.has_csa && ratio < (1 << 24)) fail("the CSA remote branch (csa.temporal_compression) is not served natively");
  m.gdn_heads = cfg_int(f, "gdn.qk_heads", 8);
  m.gdn_dim = cfg_int(f, "gdn.qk_head_dim", 64);
  const int gdn_v = cfg_int(f, "gdn.value_head_dim", 64);
  const int gdn_vh = cfg_int(f, "gdn.value_heads", m.gdn_heads);
  if (m.has_gdn && (m.gdn_dim != 64 || gdn_v != 64 || gdn_vh != m.gdn_heads ||
                    cfg_int(f, "gdn.conv_kernel", 4) != 4))
    fail("GDN blocks are served natively with 64-wide keys and values, equal head counts and conv_kernel 4");
  m.n_experts = cfg_int(f, "moe.routed_experts", 16);
  m.top_k = cfg_int(f, "moe.routed_top_k", 2);
  m.ffn = cfg_int(f, "moe.expert_hidden", 1024);
  if (m.vocab <= 0 || m.d <= 0 || m.num_loops <= 0) throw std::runtime_error("invalid model dimensions");
  // the persistent step's limits (decode_persistent.cu)
  const int D = m.d;
  if (D % 64 || D > 1024 || m.ffn % 128 || m.ffn > 2048 || m.ffn <= 0 || m.n_experts <= 0 ||
      m.n_experts > 64 || m.top_k <= 0 || m.top_k > 8 || m.top_k > m.n_experts)
    fail("d_model / expert sizes outside the persistent step's limits");
  if (m.has_csa && (m.csa_head_dim != 64 || m.csa_heads <= 0 || m.csa_heads > 16 ||
                    m.csa_heads * 64 > 1024 || m.window <= 0 || m.window > 1024))
    fail("CSA sizes outside the persistent step's limits");
  if (m.has_gdn && (m.gdn_heads <= 0 || m.gdn_heads * 64 > 1024))
    fail("GDN sizes outside the persistent step's limits");
}

void load_weights(const LlmyFile& f, llmy_model& m) {
  const int D = m.d, V = m.vocab, E = m.n_experts, F = m.ffn;
  m.embed = m.upload(as_bf16(expect(f, "embed_tokens.weight", {V, D})));
  m.stream_seed = m.upload(as_f32(expect(f, "stream_seed", {1, D})));
  m.collapse = m.upload(as_bf16(expect(f, "mhc_collapse.weight", {D, D})));
  m.final_norm = m.upload(as_f32(expect(f, "final_norm.weight", {D})));
  std::vector<llmyb_pblock> blocks(m.n_blocks);
  std::vector<void*> temps;
  auto temp = [&](size_t bytes) {
    void* p = nullptr;
    check(cudaMalloc(&p, bytes), "cudaMalloc");
    temps.push_back(p);
    return p;
  };
  try {
    for (int j = 0; j < m.n_blocks; ++j) {
      const std::string p = "recurrent_core." + std::to_string(j) + ".";
      llmyb_pblock& b = blocks[j];
      std::memset(&b, 0, sizeof(b));
      b.kind = m.kinds[j];
      std::vector<float> ffn_norm = as_f32(expect(f, p + "ffn_norm.weight", {D}));
      b.mixer_norm = m.upload(as_f32(expect(f, p + "mixer_norm.weight", {D})));
      b.ffn_norm = m.upload(ffn_norm);
      std::vector<float> router = as_f32(expect(f, p + "moe.router.logits.weight", {E, D}));
      const std::vector<float> rnorm = as_f32(expect(f, p + "moe.router.norm.weight", {D}));
      for (int e = 0; e < E; ++e)
        for (int i = 0; i < D; ++i) router[static_cast<size_t>(e) * D + i] *= ffn_norm[i] * rnorm[i];
      b.router_fold = m.upload(router);
      // experts
      const std::vector<uint16_t> gate = expert_stack(f, p, "gate_proj", E, F, D);
      const std::vector<uint16_t> up = expert_stack(f, p, "up_proj", E, F, D);
      void* g_dev = temp(gate.size() * 2);
      void* u_dev = temp(up.size() * 2);
      check(cudaMemcpy(g_dev, gate.data(), gate.size() * 2, cudaMemcpyHostToDevice), "upload");
      check(cudaMemcpy(u_dev, up.data(), up.size() * 2, cudaMemcpyHostToDevice), "upload");
      void* w13 = m.alloc(static_cast<size_t>(E) * 2 * F * D * 2);
      check_status(llmyb_moe_pack_w13(g_dev, u_dev, E, F, D, w13, nullptr), "llmyb_moe_pack_w13");
      b.w13 = w13;
      b.w2 = m.upload(expert_stack(f, p, "down_proj", E, D, F));
      if (b.kind == 0) {
        const int HD = m.csa_heads * m.csa_head_dim;
        const FileTensor& out = f.tensor(p + "mixer.out.weight");
        const FileTensor& lo = f.tensor(p + "mixer.local_out.weight");
        if (out.shape.size() != 2 || lo.shape.size() != 2 || out.shape[0] != D ||
            out.shape[1] != lo.shape[0])
          throw std::runtime_error(p + "mixer.out / local_out shapes do not chain");
        const int A = static_cast<int>(out.shape[1]), Dv = static_cast<int>(lo.shape[1]);
        const FileTensor& val = expect(f, p + "mixer.value.weight", {Dv, D});
        // W_o = bf16(out . local_out); value rows = bf16(W_o . value) (fp32 products)
        const std::vector<float> out32 = as_f32(out), lo32 = as_f32(lo);
        std::vector<float> v32 = as_f32(val);
        for (float& x : v32) {  // the value weight as the model stores it (bf16)
          const uint32_t u = static_cast<uint32_t>(float_to_bf16(x)) << 16;
          std::memcpy(&x, &u, 4);
        }
        float* a_d = static_cast<float*>(temp(out32.size() * 4));
        float* b_d = static_cast<float*>(temp(lo32.size() * 4));
        float* wo_d = static_cast<float*>(temp(static_cast<size_t>(D) * Dv * 4));
        float* v_d = static_cast<float*>(temp(v32.size() * 4));
        float* wvo_d = static_cast<float*>(temp(static_cast<size_t>(D) * D * 4));
        check(cudaMemcpy(a_d, out32.data(), out32.size() * 4, cudaMemcpyHostToDevice), "upload");
        check(cudaMemcpy(b_d, lo32.data(), lo32.size() * 4, cudaMemcpyHostToDevice), "upload");
        check(cudaMemcpy(v_d, v32.data(), v32.size() * 4, cudaMemcpyHostToDevice), "upload");
        const dim3 tb(16, 16);
        fold_matmul_kernel<<<dim3((Dv + 15) / 16, (D + 15) / 16), tb>>>(a_d, b_d, wo_d, D, A, Dv);
        round_bf16_kernel<<<64, 256>>>(wo_d, nullptr, static_cast<int64_t>(D) * Dv);
        fold_matmul_kernel<<<dim3((D + 15) / 16, (D + 15) / 16), tb>>>(wo_d, v_d, wvo_d, D, Dv, D);
        check(cudaGetLastError(), "fold kernels");
        const int rows = 2 * HD + D;
        __nv_bfloat16* w_in = static_cast<__nv_bfloat16*>(m.alloc(static_cast<size_t>(rows) * D * 2));
        const std::vector<uint16_t> q = as_bf16(expect(f, p + "mixer.query.weight", {HD, D}));
        const std::vector<uint16_t> k = as_bf16(expect(f, p + "mixer.key.weight", {HD, D}));
        check(cudaMemcpy(w_in, q.data(), q.size() * 2, cudaMemcpyHostToDevice), "upload");
        check(cudaMemcpy(w_in + static_cast<size_t>(HD) * D, k.data(), k.size() * 2,
                         cudaMemcpyHostToDevice), "upload");
        round_bf16_kernel<<<64, 256>>>(wvo_d, w_in + static_cast<size_t>(2 * HD) * D,
                                       static_cast<int64_t>(D) * D);
        check(cudaGetLastError(), "fold kernels");
        b.w_in = w_in;
        b.rows = rows;
      } else {
        const int H = m.gdn_heads, HK = H * 64;
        std::vector<uint16_t> w;
        const char* names[5] = {"q_proj", "k_proj", "v_proj", "gate_proj", "beta_proj"};
        const int rows_of[5] = {HK, HK, HK, HK, H};
        for (int i = 0; i < 5; ++i) {
          const std::vector<uint16_t> part =
              as_bf16(expect(f, p + "mixer." + names[i] + ".weight", {rows_of[i], D}));
          w.insert(w.end(), part.begin(), part.end());
        }
        int rows = 4 * HK + H;
        const int pad = (8 - rows % 8) % 8;
        w.resize(static_cast<size_t>(rows + pad) * D, 0);
        rows += pad;
        b.w_in = m.upload(w);
        b.rows = rows;
        b.beta_bias = m.upload(as_f32(expect(f, p + "mixer.beta_proj.bias", {H})));
        b.decay_logit = m.upload(as_f32(expect(f, p + "mixer.decay_logit", {H})));
        b.w_out = m.upload(as_bf16(expect(f, p + "mixer.out_proj.weight", {D, HK})));
        const FileTensor& conv = f.tensor(p + "mixer.conv.weight");
        if (conv.numel() != static_cast<int64_t>(D) * 4)
          throw std::runtime_error(p + "mixer.conv.weight has shape " + shape_str(conv.shape) +
                                   ", expected [" + std::to_string(D) + ", 1, 4]");
        b.conv = m.upload(as_f32(conv));
      }
      m.max_rows = std::max(m.max_rows, b.rows);
      check(cudaDeviceSynchronize(), "load");
      for (void* t : temps) cudaFree(t);
      temps.clear();
    }
  } catch (...) {
    for (void* t : temps) cudaFree(t);
    throw;
  }
  m.blocks = m.upload(blocks);
}

void check_grid(const llmy_model& m) {
  const int g = m.grid;
  if (g <= 0) throw std::runtime_error("the persistent decode step does not fit this device");
  if (m.d > g * 16 || m.max_rows > 2 * g * 16 ||
      (m.has_csa && (m.d / 8 > g || (m.window + 15) / 16 > g)) ||
      (m.has_gdn && m.gdn_heads * 2 > g))
    throw std::runtime_error("the model is too wide for " + std::to_string(g) +
                             " persistent CTAs on this device");
}

llmy_state* new_state(llmy_model* m) {
  auto s = std::make_unique<llmy_state>();
  s->m = m;
  s->loops = m->num_loops;
  const int D = m->d, nb = m->n_blocks, nl = s->loops, G = m->grid;
  std::vector<llmyb_player> layers(static_cast<size_t>(nl) * nb);
  for (int i = 0; i < nl; ++i)
    for (int j = 0; j < nb; ++j) {
      llmyb_player& l = layers[static_cast<size_t>(i) * nb + j];
      std::memset(&l, 0, sizeof(l));
      if (m->kinds[j] == 0) {
        const size_t hd = static_cast<size_t>(m->csa_heads) * m->csa_head_dim;
        l.ring_k = s->alloc(static_cast<size_t>(m->window) * hd * 2, true);
        l.ring_v = s->alloc(static_cast<size_t>(m->window) * D * 2, true);
      } else {
        l.gdn_state = static_cast<float*>(
            s->alloc(static_cast<size_t>(m->gdn_heads) * 64 * 64 * 4, true));
        l.conv_hist = s->alloc(static_cast<size_t>(3) * D * 2, true);
      }
    }
  void* layers_dev = s->alloc(layers.size() * sizeof(llmyb_player));
  check(cudaMemcpy(layers_dev, layers.data(), layers.size() * sizeof(llmyb_player),
                   cudaMemcpyHostToDevice), "upload");
  s->io = static_cast<int64_t*>(s->alloc(16, true));
  check(cudaMallocHost(&s->io_host, 16), "cudaMallocHost");
  check(cudaMallocHost(&s->status_host, 4), "cudaMallocHost");
  llmyb_pdecode& p = s->p;
  std::memset(&p, 0, sizeof(p));
  p.d_model = D;
  p.n_blocks = nb;
  p.n_loops = nl;
  p.vocab = m->vocab;
  p.csa_heads = m->has_csa ? m->csa_heads : 0;
  p.csa_head_dim = m->csa_head_dim;
  p.window = m->window;
  p.gdn_heads = m->has_gdn ? m->gdn_heads : 0;
  p.gdn_dim = m->gdn_dim;
  p.n_experts = m->n_experts;
  p.top_k = m->top_k;
  p.ffn = m->ffn;
  p.eps = 1e-6f;  // RMSNorm epsilon of the model (model/layers/norms.py; model.cpp:1925)
  p.grid = G;
  p.blocks = m->blocks;
  p.layers = static_cast<const llmyb_player*>(layers_dev);
  p.embed = m->embed;
  p.stream_seed = m->stream_seed;
  p.collapse = m->collapse;
  p.final_norm = m->final_norm;
  p.token = s->io;
  p.positions = reinterpret_cast<int32_t*>(s->io + 1);
  const int hc = std::max(m->csa_heads, 1), w = std::max(m->window, 1);
  p.x = static_cast<float*>(s->alloc(static_cast<size_t>(2) * D * 4));
  p.proj = s->alloc(static_cast<size_t>(m->max_rows) * 2);
  p.normed = s->alloc(static_cast<size_t>(D) * 2);
  p.scores = static_cast<float*>(s->alloc(static_cast<size_t>(hc) * w * 4));
  p.stats = static_cast<float*>(s->alloc(static_cast<size_t>(G) * hc * 2 * 4));
  p.mix = s->alloc(static_cast<size_t>(std::max(D, m->gdn_heads * 64)) * 2);
  p.partials = static_cast<float*>(s->alloc(static_cast<size_t>(G) * (2 + m->n_experts) * 4));
  p.hbuf = s->alloc(static_cast<size_t>(m->top_k) * m->ffn * 2);
  p.ybuf = s->alloc(static_cast<size_t>(m->top_k) * D * 2);
  p.collapsed = s->alloc(static_cast<size_t>(D) * 2);
  p.route_idx = static_cast<int32_t*>(s->alloc(static_cast<size_t>(nl) * nb * m->top_k * 4));
  p.route_prob = static_cast<float*>(s->alloc(static_cast<size_t>(nl) * nb * m->top_k * 4));
  p.logits = static_cast<float*>(s->alloc(static_cast<size_t>(m->vocab) * 4));
  p.bar = static_cast<uint32_t*>(s->alloc(8));
  p.status = static_cast<int32_t*>(s->alloc(4));
  p.head_part = static_cast<float*>(s->alloc(static_cast<size_t>(G) * 4 * 4));
  return s.release();
}

int loops_for(const llmy_model* m, const llmy_state* s, int32_t requested, const char* who) {
  int loops = requested > 0 ? requested : m->num_loops;
  loops = std::min(loops, m->num_loops);
  if (loops > s->loops) {
    std::fprintf(stderr, "[%s] the state holds %d loops, %d requested: running %d\n", who,
                 s->loops, loops, s->loops);
    loops = s->loops;
  }
  return loops;
}

// Launch one step; returns false (after printing why) if the launch failed.
bool launch(llmy_state* s, const int64_t* token_dev, int loops, bool skip_head, const char* who) {
  s->p.token = token_dev;
  s->p.n_loops = loops;
  s->p.skip_head = skip_head ? 1 : 0;
  const int32_t st = llmyb_decode_persistent(&s->p, nullptr);
  if (st != 0) {
    std::fprintf(stderr, "[%s] decode step launch failed with status %d\n", who, st);
    return false;
  }
  return true;
}

// Copy the logits out, read the device status word and wait for the stream.
void finish(llmy_state* s, float* logits_out, const char* who) {
  const llmy_model* m = s->m;
  cudaError_t e = cudaSuccess;
  if (logits_out)
    e = cudaMemcpyAsync(logits_out, s->p.logits, static_cast<size_t>(m->vocab) * 4,
                        cudaMemcpyDefault, nullptr);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(s->status_host, s->p.status, 4, cudaMemcpyDeviceToHost, nullptr);
  if (e == cudaSuccess) e = cudaStreamSynchronize(nullptr);
  if (e != cudaSuccess) {
    std::fprintf(stderr, "[%s] %s\n", who, cudaGetErrorString(e));
    return;
  }
  if (*s->status_host != 0) {
    std::fprintf(stderr, "[%s] device status %d%s\n", who, *s->status_host,
                 *s->status_host == LLMYB_ETIMEOUT ? " (a grid barrier timed out)" : "");
    cudaMemsetAsync(s->p.status, 0, 4, nullptr);
    cudaStreamSynchronize(nullptr);
  }
}

}  // namespace

// ---------------------------------------------------------------- C API
LLMYB_API llmy_model* llmy_load(const char* path) {
  try {
    if (!path) throw std::runtime_error("null path");
    auto m = std::make_unique<llmy_model>();
    LlmyFile f(path);
    load_config(f, *m);
    check(cudaGetDevice(&m->device), "cudaGetDevice");
    m->grid = llmyb_decode_persistent_grid();
    if (m->grid <= 0)
      throw std::runtime_error("the persistent decode step does not fit this device (status " +
                               std::to_string(-m->grid) + ")");
    load_weights(f, *m);
    check_grid(*m);
    return m.release();
  } catch (const std::exception& e) {
    std::fprintf(stderr, "[llmy_load] %s\n", e.what());
    return nullptr;
  }
}

LLMYB_API void llmy_free(llmy_model* m) {
  if (!m) return;
  cudaDeviceSynchronize();
  delete m;
}

LLMYB_API int32_t llmy_vocab_size(const llmy_model* m) { return m ? m->vocab : 0; }
LLMYB_API int32_t llmy_d_model(const llmy_model* m) { return m ? m->d : 0; }
LLMYB_API int32_t llmy_num_loops(const llmy_model* m) { return m ? m->num_loops : 0; }
LLMYB_API int32_t llmy_max_loops(const llmy_model* m) { return m ? m->num_loops : 0; }
LLMYB_API int32_t llmy_mhc_streams(const llmy_model* m) { return m ? 1 : 0; }

LLMYB_API void llmy_set_num_loops(llmy_model* m, int32_t n) {
  if (m && n >= 1) m->num_loops = n;
}

LLMYB_API void llmy_set_fixed_loops(llmy_model* m, int32_t n) {
  if (m && n >= 1) m->num_loops = n;
}

LLMYB_API llmy_state* llmy_state_new(llmy_model* m) {
  try {
    if (!m) throw std::runtime_error("null model");
    return new_state(m);
  } catch (const std::exception& e) {
    std::fprintf(stderr, "[llmy_state_new] %s\n", e.what());
    return nullptr;
  }
}

LLMYB_API void llmy_state_free(llmy_state* s) {
  if (!s) return;
  cudaDeviceSynchronize();
  delete s;
}

LLMYB_API void llmy_state_reset(llmy_state* s) {
  if (!s) return;
  for (auto& r : s->recurrent) cudaMemsetAsync(r.first, 0, r.second, nullptr);
  cudaStreamSynchronize(nullptr);
  s->last_executed_loops = 0;
}

LLMYB_API void llmy_prefill(llmy_model* m, llmy_state* s, const int32_t* tokens,
                            int32_t n_tokens, float* logits_out) {
  if (!m || !s || s->m != m) {
    std::fprintf(stderr, "[llmy_prefill] null or mismatched model / state handle\n");
    return;
  }
  if (n_tokens <= 0) return;
  if (!tokens) {
    std::fprintf(stderr, "[llmy_prefill] null tokens\n");
    return;
  }
  if (n_tokens > s->prompt_cap) {
    void* p = nullptr;
    if (cudaMalloc(&p, static_cast<size_t>(n_tokens) * 8) != cudaSuccess) {
      std::fprintf(stderr, "[llmy_prefill] cannot allocate %d prompt ids\n", n_tokens);
      return;
    }
    if (s->prompt) {
      cudaFree(s->prompt);
      s->allocs.erase(std::find(s->allocs.begin(), s->allocs.end(), s->prompt));
    }
    s->prompt = static_cast<int64_t*>(p);
    s->allocs.push_back(p);
    s->prompt_cap = n_tokens;
  }
  // a host or device token array: gather it to the host as int64 ids
  std::vector<int32_t> t32(static_cast<size_t>(n_tokens));
  if (cudaMemcpy(t32.data(), tokens, t32.size() * 4, cudaMemcpyDefault) != cudaSuccess) {
    std::fprintf(stderr, "[llmy_prefill] cannot read the tokens\n");
    return;
  }
  const std::vector<int64_t> t64(t32.begin(), t32.end());
  cudaMemcpy(s->prompt, t64.data(), t64.size() * 8, cudaMemcpyHostToDevice);
  cudaMemsetAsync(s->p.positions, 0, 4, nullptr);  // positions 0 .. n-1 (model.cpp:1962-1965)
  const int loops = loops_for(m, s, 0, "llmy_prefill");
  for (int32_t i = 0; i < n_tokens; ++i)
    if (!launch(s, s->prompt + i, loops, i != n_tokens - 1, "llmy_prefill")) return;
  s->last_executed_loops = loops;
  finish(s, logits_out, "llmy_prefill");
}

LLMYB_API void llmy_decode(llmy_model* m, llmy_state* s, int32_t token, int32_t position,
                           int32_t num_loops, float* logits_out) {
  if (!m || !s || s->m != m) {
    std::fprintf(stderr, "[llmy_decode] null or mismatched model / state handle\n");
    return;
  }
  const int loops = loops_for(m, s, num_loops, "llmy_decode");
  // the pinned slot is free: the previous step's finish() waited for the stream
  s->io_host[0] = token;
  int32_t pos32[2] = {position, 0};
  std::memcpy(&s->io_host[1], pos32, 8);
  if (cudaMemcpyAsync(s->io, s->io_host, 16, cudaMemcpyHostToDevice, nullptr) != cudaSuccess) {
    std::fprintf(stderr, "[llmy_decode] cannot stage the token\n");
    return;
  }
  if (!launch(s, s->io, loops, false, "llmy_decode")) return;
  s->last_executed_loops = loops;
  finish(s, logits_out, "llmy_decode");
}

LLMYB_API int32_t llmy_sample(const float* logits, int32_t vocab_size, float temperature,
                              int32_t top_k, float top_p, float repetition_penalty,
                              const int32_t* recent_tokens, int32_t n_recent,
                              uint64_t* rng_state) {
  return llmyb_engine_sample(logits, vocab_size, temperature, top_k, top_p, repetition_penalty,
                             recent_tokens, n_recent, rng_state);
}

LLMYB_API int32_t llmyb_engine_routes(const llmy_state* s, int32_t* idx, float* prob,
                                      int32_t capacity) {
  if (!s || !idx || capacity < 0) return -LLMYB_EINVAL;
  const int32_t n = s->last_executed_loops * s->m->n_blocks * s->m->top_k;
  if (n > capacity) return -LLMYB_EINVAL;
  cudaError_t e = cudaMemcpy(idx, s->p.route_idx, static_cast<size_t>(n) * 4, cudaMemcpyDefault);
  if (e == cudaSuccess && prob)
    e = cudaMemcpy(prob, s->p.route_prob, static_cast<size_t>(n) * 4, cudaMemcpyDefault);
  return e == cudaSuccess ? n : -static_cast<int32_t>(e);
}

LLMYB_API int32_t llmy_last_executed_loops(const llmy_state* s) {
  return s ? s->last_executed_loops : 0;
}

LLMYB_API void llmy_sync(void) { cudaDeviceSynchronize(); }

LLMYB_API int32_t llmy_mhc_sinkhorn4(const float* input, float* output, int32_t matrices,
                                     int32_t iterations, void* stream) {
  return llmyb_mhc_sinkhorn4(input, output, matrices, iterations, stream);
}

LLMYB_API int32_t llmy_moe_selected_fp32(const float* x, const int64_t* idx, const float* prob,
                                         const float* gate_up, const float* down,
                                         float* activation, float* route_output, float* out,
                                         int32_t D, int32_t H, int32_t E, int32_t k,
                                         void* stream) {
  return llmyb_moe_selected_fp32(x, idx, prob, gate_up, down, activation, route_output, out, D,
                                 H, E, k, stream);
}
