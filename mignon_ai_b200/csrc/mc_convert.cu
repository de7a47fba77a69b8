// quant.Quantize (internal/quant/convert.go:8-98) of a full-precision model file, on the device.
//
// The file is binfmt kind 1 (internal/checkpoint/checkpoint.go:86-94): "MGNN", version 1, kind 1,
// the JSON of File{Vocab, Merges, Metadata} without weights, then one float32 array holding every
// parameter in the order of ca.NewLayout (internal/ca/layout.go:103-161). The architecture comes
// from the metadata as pkg/model.Decode builds it (pkg/model/model.go:85-103): vocabulary = the
// tokenizer's entries, blocks = ca.BuildBlockConfigs (internal/ca/model.go:33-59).
//
// The weight vector is uploaded once; one kernel takes max|w| of every matrix, a second rounds it
// to int8 (NewTensorF32, internal/quant/tensor.go:12-42). Biases, gains and norms are copied on
// the host. The result is the HostModel an INT8 file of the same model would give.

namespace mc {
namespace eng {

// One matrix of quant.Quantize: rows x cols weights starting at src of the flat vector, rows
// `stride` apart (stride > cols where each row carries its bias after its weights), into dst.
struct QuantMatrix {
  unsigned long long src, dst;
  int rows, cols, stride;
};

// max |w| of matrix blockIdx.y; the bit patterns of non-negative floats order like their values.
__global__ void quant_maxabs_kernel(const float* w, const QuantMatrix* mats, unsigned int* maxbits) {
  const QuantMatrix q = mats[blockIdx.y];
  const size_t n = (size_t)q.rows * q.cols;
  float m = 0.f;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const size_t r = i / q.cols, c = i - r * q.cols;
    m = fmaxf(m, fabsf(w[q.src + r * q.stride + c]));
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) atomicMax(&maxbits[blockIdx.y], __float_as_uint(m));
}

// NewTensorF32: scale = max|w| / 127 in float32, q = round(w / scale) half away from zero,
// clamped to [-127, 127]; an all-zero matrix gets scale 1 and zeros.
__global__ void quant_round_kernel(const float* w, const QuantMatrix* mats, const unsigned int* maxbits, int8_t* out,
                                   float* scales) {
  const QuantMatrix q = mats[blockIdx.y];
  const float mx = __uint_as_float(maxbits[blockIdx.y]);
  const float scale = mx == 0.f ? 1.f : __fdiv_rn(mx, 127.0f);
  if (blockIdx.x == 0 && threadIdx.x == 0) scales[blockIdx.y] = scale;
  const size_t n = (size_t)q.rows * q.cols;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const size_t r = i / q.cols, c = i - r * q.cols;
    int8_t v = 0;
    if (mx != 0.f) {
      const float x = roundf(__fdiv_rn(w[q.src + r * q.stride + c], scale));
      v = (int8_t)fminf(fmaxf(x, -127.f), 127.f);
    }
    out[q.dst + i] = v;
  }
}

}  // namespace eng

namespace {

uint32_t rd_u32(const uint8_t* p) {
  return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}

}  // namespace

// Parses a full-precision model file and quantizes it on `device` into m. max_context <= 0 takes
// the metadata's context size (pkg/model normalizes a missing one to 64, model.go:25 / :123-131).
int quantize_full_model(const uint8_t* data, size_t n, int max_context, int device, HostModel& m) {
  using namespace eng;
  if (n < 12 || memcmp(data, "MGNN", 4)) return set_error(kBadModel, "not a binary model file");
  if ((data[4] | (data[5] << 8)) != 1) return set_error(kBadModel, "binary model file version is not supported");
  if (data[6] != 1) return set_error(kBadModel, "not a full-precision model file");
  const uint32_t hlen = rd_u32(data + 8);
  if ((uint64_t)hlen + 16 > n) return set_error(kBadModel, "full-precision model file is truncated");
  json::Parser p(reinterpret_cast<const char*>(data) + 12, hlen);
  auto root = p.parse();
  if (!root || root->type != json::Value::Obj) return set_error(kBadModel, "malformed model header JSON");
  const json::Value* vocab = root->get("vocab");
  const json::Value* meta = root->get("metadata");
  if (!vocab || vocab->type != json::Value::Arr || vocab->items.empty())
    return set_error(kBadModel, "model file holds no tokenizer");
  if (!meta || meta->type != json::Value::Obj) return set_error(kBadModel, "model file lacks architecture metadata");
  const long V = (long)vocab->items.size();
  const long D = (long)meta->number("state_size", 0), H = (long)meta->number("hidden_size", 0);
  const int nblocks = (int)meta->number("blocks", 0), steps = (int)meta->number("steps", 0);
  const int base = (int)meta->number("dilation_base", 0);
  const json::Value* te = meta->get("tied_embed");
  const bool tied = te && te->type == json::Value::Bool && te->b;
  const int heads = (int)meta->number("attn_heads", 0), window = (int)meta->number("attn_window", 0);
  if (D < 1 || H < 1 || steps < 1 || nblocks < 1)
    return set_error(kBadModel, "model file lacks architecture metadata (state_size, hidden_size, steps, blocks)");
  if (nblocks > 4096 || D > 65536 || H > 65536) return set_error(kBadModel, "model shape out of range");
  int ctx = max_context;
  if (ctx <= 0) ctx = (int)meta->number("context_size", 0);
  if (ctx <= 0) ctx = 64;

  // ca.BuildBlockConfigs, then NewLayout's defaults (base <= 1 -> 2, initial dilation < 1 -> 1)
  struct Cfg {
    int steps, base, init;
  };
  std::vector<Cfg> cfg;
  if (nblocks == 2 && (steps == 3 || steps == 5) && base == 2) {
    cfg = {{3, 2, 1}, {3, 2, 4}};  // DefaultTwoBlockConfig (internal/ca/model.go:25-30)
  } else {
    int cur = 1;
    for (int b = 0; b < nblocks; ++b) {
      cfg.push_back({steps, base, cur});
      for (int s = 0; s < steps - 1 && nblocks > 1; ++s) {
        cur *= base;
        if (cur > 32) {  // MaxCADilation (internal/ca/config.go:59)
          cur = 32;
          break;
        }
      }
    }
  }
  for (Cfg& c : cfg) {
    if (c.base <= 1) c.base = 2;
    if (c.init < 1) c.init = 1;
  }

  // ca.NewLayout offsets
  const long in_dim = 3 * D, l1 = 2 * H * (in_dim + 1), l2 = 2 * D * (H + 1);
  struct BOff {
    long l1, l2, gamma, sel, attn;
  };
  std::vector<BOff> off;
  long cur = V * D;
  for (size_t b = 0; b < cfg.size(); ++b) {
    const long sel = cur + l1 + l2 + D;
    long extra = sel + D * D, attn = -1;
    if (heads > 0) {
      attn = extra;
      extra += D + 4 * D * D;
    }
    off.push_back({cur, cur + l1, cur + l1 + l2, sel, attn});
    cur = extra;
  }
  const long final_norm = cur;
  cur += D;
  const long head = cur;
  const long total = cur + (tied ? V : V * (D + 1));

  // the weight array
  const uint8_t* rest = data + 12 + hlen;
  const size_t rest_n = n - 12 - hlen;
  const uint32_t cnt = rd_u32(rest);
  if ((uint64_t)cnt * 4 + 4 != rest_n) return set_error(kBadModel, "full-precision model file: weight array size mismatch");
  if ((long)cnt != total)
    return set_error(kBadModel, "architecture mismatch: file has " + std::to_string(cnt) + " weights, the model needs " +
                                    std::to_string(total));
  std::vector<float> w(cnt);
  memcpy(w.data(), rest + 4, (size_t)cnt * 4);

  // the matrices, in HostModel order
  std::vector<QuantMatrix> mats;
  std::vector<HostTensor*> dst;
  unsigned long long out_n = 0;
  auto add = [&](long src, long rows, long cols, long stride, HostTensor* t) {
    mats.push_back({(unsigned long long)src, out_n, (int)rows, (int)cols, (int)stride});
    dst.push_back(t);
    out_n += (unsigned long long)rows * cols;
  };
  m = HostModel();
  m.vocab = (int)V;
  m.state = (int)D;
  m.hidden = (int)H;
  m.tied = tied;
  m.context_size = ctx;
  m.attn_heads = heads;
  m.attn_window = window;
  m.blocks.resize(cfg.size());
  add(0, 1, V * D, V * D, &m.embed);
  for (size_t b = 0; b < cfg.size(); ++b) {
    HostBlock& bl = m.blocks[b];
    const BOff& o = off[b];
    bl.steps = cfg[b].steps;
    bl.dilation_base = cfg[b].base;
    bl.initial_dilation = cfg[b].init;
    add(o.l1, 2 * H, in_dim, in_dim + 1, &bl.w1);
    bl.b1.resize(2 * H);
    for (long h = 0; h < 2 * H; ++h) bl.b1[h] = w[o.l1 + h * (in_dim + 1) + in_dim];
    add(o.l2, 2 * D, H, H + 1, &bl.w2);
    bl.b2.resize(2 * D);
    for (long s = 0; s < 2 * D; ++s) bl.b2[s] = w[o.l2 + s * (H + 1) + H];
    bl.gamma.assign(w.begin() + o.gamma, w.begin() + o.gamma + D);
    add(o.sel, 1, D * D, D * D, &bl.wsel);
    if (o.attn >= 0) {
      bl.has_attn = true;
      bl.attn_norm.assign(w.begin() + o.attn, w.begin() + o.attn + D);
      add(o.attn + D, 1, 3 * D * D, 3 * D * D, &bl.qkv);
      add(o.attn + D + 3 * D * D, 1, D * D, D * D, &bl.out);
    }
  }
  m.final_norm.assign(w.begin() + final_norm, w.begin() + final_norm + D);
  if (tied) {
    m.head_b.assign(w.begin() + head, w.begin() + head + V);
  } else {
    add(head, V, D, D + 1, &m.head_w);
    m.head_b.resize(V);
    for (long v = 0; v < V; ++v) m.head_b[v] = w[head + v * (D + 1) + D];
  }
  for (const QuantMatrix& q : mats)
    if ((long)q.rows * q.cols > (1L << 31) - 1) return set_error(kUnsupported, "matrix too large to quantize");

  // on the device: upload, max |w|, round, read back
  MC_CUDA(cudaSetDevice(device));
  const size_t nm = mats.size();
  const size_t bytes = (size_t)cnt * 4 + nm * sizeof(QuantMatrix) + nm * 8 + out_n + 1024;
  DevBuf buf;
  if (cudaMalloc(&buf.p, bytes) != cudaSuccess) {
    cudaGetLastError();
    return set_error(kOutOfMemory, "cudaMalloc failed while quantizing a full-precision model");
  }
  char* q = static_cast<char*>(buf.p);
  float* d_w = reinterpret_cast<float*>(q);
  q += ((size_t)cnt * 4 + 255) & ~(size_t)255;
  QuantMatrix* d_mats = reinterpret_cast<QuantMatrix*>(q);
  q += (nm * sizeof(QuantMatrix) + 255) & ~(size_t)255;
  unsigned int* d_max = reinterpret_cast<unsigned int*>(q);
  float* d_scale = reinterpret_cast<float*>(d_max + nm);
  q += (nm * 8 + 255) & ~(size_t)255;
  int8_t* d_out = reinterpret_cast<int8_t*>(q);
  cudaStream_t s = 0;
  MC_CUDA(cudaMemcpyAsync(d_w, w.data(), (size_t)cnt * 4, cudaMemcpyHostToDevice, s));
  MC_CUDA(cudaMemcpyAsync(d_mats, mats.data(), nm * sizeof(QuantMatrix), cudaMemcpyHostToDevice, s));
  MC_CUDA(cudaMemsetAsync(d_max, 0, nm * 4, s));
  const dim3 grid(148, (unsigned)nm);
  quant_maxabs_kernel<<<grid, 256, 0, s>>>(d_w, d_mats, d_max);
  MC_CUDA(cudaGetLastError());
  quant_round_kernel<<<grid, 256, 0, s>>>(d_w, d_mats, d_max, d_out, d_scale);
  MC_CUDA(cudaGetLastError());
  std::vector<int8_t> out(out_n);
  std::vector<float> scales(nm);
  MC_CUDA(cudaMemcpyAsync(out.data(), d_out, out_n, cudaMemcpyDeviceToHost, s));
  MC_CUDA(cudaMemcpyAsync(scales.data(), d_scale, nm * 4, cudaMemcpyDeviceToHost, s));
  MC_CUDA(cudaStreamSynchronize(s));
  for (size_t i = 0; i < nm; ++i) {
    const size_t len = (size_t)mats[i].rows * mats[i].cols;
    dst[i]->data.assign(out.begin() + mats[i].dst, out.begin() + mats[i].dst + len);
    dst[i]->scale = scales[i];
  }
  return kOk;
}

}  // namespace mc

extern "C" int mc_load_model_full(mc_ctx* ctx, const uint8_t* data, size_t n, int max_context, mc_model** out) {
  clear_error();
  DeviceRestore restore_device;
  if (!ctx || !data || !out || ctx->devices.empty()) return set_error(kInvalidArgument, "mc_load_model_full: null argument");
  auto m = std::make_unique<mc_model>();
  m->ctx = ctx;
  int st = quantize_full_model(data, n, max_context, ctx->devices[0], m->host);
  if (st != kOk) return st;
  for (int d : ctx->devices) {
    std::unique_ptr<DevModel> dm;
    if ((st = build_dev_model(m->host, d, dm)) != kOk) return st;
    m->dev.push_back(std::move(dm));
  }
  *out = m.release();
  return kOk;
}
