// Shared definitions of the engine kernels: tile geometry, the pre-tiled weight image, the
// per-launch argument blocks and the reference's scalar functions.
#pragma once
#include "mc_sm100.cuh"

namespace mc {
namespace eng {

constexpr int kRows = 128;                 // rows per tile (TMEM lanes)
constexpr int kTile = 128 * 128;           // one 128 x 128 int8 operand tile (16 KB)
constexpr int kASlots = 3;                 // activation slots, three digit planes each
constexpr int kASlot = 3 * kTile;          // 48 KB
constexpr int kBStages = 4;                // weight-tile ring
constexpr int kNC = 128;                   // output columns per chunk (MMA N)
constexpr int kMaxSteps = 8;
constexpr int kMaxGemms = 2 + 3 * kMaxSteps;
constexpr int kMaxStops = 8;               // stop tokens of a generation
constexpr int kHalfChunk = 64;             // paired chunks: 64 value/delta + 64 gate columns

// Pre-tiled weight image (built at model load): for output chunk c and K tile kt, a 16 KB tile
// whose row r holds weight row perm[c*128 + r] (zeros past the end), bytes [kt*128, kt*128+128)
// of it (zeros past K), in the 128-byte swizzled K-major layout. Tile (c, kt) starts at byte
// (c * ktiles + kt) * kTile.

enum GemmType : int { kGOut = 0, kGWsel = 1, kGW1 = 2, kGW2 = 3, kGQkv = 4, kGHead = 5 };

struct GemmSpec {
  const uint8_t* tiles;
  int K, ktiles, nchunks, type, step;
  float scale;
};

// One launch of the block kernel: rows of a tile are `spt` session slots of P rows each (row r:
// slot r / P, in-segment position t = r % P); decode is P = 1, spt = 128.
struct BlockArgs {
  int P, spt, n_sess, n_tiles;
  const int32_t* pos0;     // [S] position of the first row of each session's segment
  const int32_t* seglen;   // [S] rows of the segment (0 = inactive)
  const int32_t* tokens;   // [S * P] token ids of the segment rows
  int D, H, V;
  int block, nsteps, bs0, ring, total_steps;
  int dil[kMaxSteps];
  int embed_first, residual, has_out, has_attn, final_norm;
  int attn_slot, n_attn, cache, window, dh;
  int ngemms;
  GemmSpec gemms[kMaxGemms];
  const int8_t* embed;
  float embed_scale;
  const float* gamma;       // [D] or null (no norm gain: the norm cell is cur itself)
  const float* b1;          // [2H]
  const float* b2;          // [2D]
  const float* latch_base;  // [D]
  const float* attn_norm;   // [D]
  const float* final_gain;  // [D] or null
  // session state
  float* norm_ring;  // [S][total_steps][ring][D]
  float* latch;      // [S][total_steps][D]
  float* kv;         // [n_attn][S][K|V][head][slot][dh]
  // scratch, indexed by global row (tile * 128 + r)
  float* cur;        // [rows][D]
  float* blockin;    // [rows][D]
  float* xbuf;       // [rows][3D]
  float* hbuf;       // [rows][H]
  float* qbuf;       // [rows][D]
  float* att;        // [rows][D]
  float* att_rowmax; // [rows]
  float* fnorm;      // [rows][D] final-norm output (final kernel)
  float* fnorm_rowmax;
  float* kvlin;      // [S][P][2][D] keys and values of a prefill segment
  unsigned long long* trace;  // optional phase timestamps of CTA 0 (null: off)
  int trace_fine;             // also time every chunk of every GEMM
  int dec_kt;                 // decode kernel: K tiles of its activation-plane region
  // block kernel: per-SM cache of the digit planes of a GEMM whose K tiles do not all fit in the
  // A slots ([SM id < a_cache_sms][K tile < a_cache_kt][3 planes x 128 x 128], or null): sliced once
  // for the GEMM's first chunk, copied back into the slots for the others
  uint8_t* a_cache;
  int a_cache_kt, a_cache_sms;
  // decode kernel, final launch with the greedy head fused in (fuse_head): the last GEMM is the
  // tied head; each session's first argmax and probability (argmaxProb) are written as
  // select_kernel would, and the last CTA to finish advances the step counter.
  int fuse_head;
  float* head_logits;   // [S][V] or null: the fused head writes each session's logits instead of
                        // selecting (the decode-loop policy reads them; no step counter advance)
  const float* head_b;  // [V]
  int32_t* next_tok;    // [S]
  int32_t* out_tok;     // [S][out_stride] or null
  float* out_prob;      // [S][out_stride] or null
  int out_stride;
  int32_t* pos_w;       // [S] positions, advanced by one
  int32_t* step;        // device step counter (output column)
  int32_t* done;        // finished-CTA counter (zero between launches)
  int n_stops;          // a chosen token among stops ends its session (seglen_w = 0, no output)
  int stops[kMaxStops];
  int32_t* seglen_w;
  const int32_t* tile_list;  // CTA i runs tile tile_list[i] (a pass over some tiles only), or null: tile tile0 + i
  int tile0;                 // first tile of a pass over a contiguous range of tiles (0: from the first)
  int32_t* gen_n;       // [S] tokens each session has emitted (its output column), or null: *step
  const int32_t* limit; // [S] tokens a session may emit (it ends after the last), with gen_n
};

// sigmoidClamped (internal/quant/stream.go:128-136): saturated beyond |x| > 15, else 1/(1+e^-x)
// with float32 add and divide. The reference rounds a float64 exp to float32 and divides exactly;
// here the exp is the fast form (ex2 of x log2 e) and the divide the fast reciprocal: for
// |x| <= 15 within 2e-6 relative of it, far inside the logit tolerance, and a fraction of the
// instructions in epilogues that are bound by their count.
__device__ __forceinline__ float sigmoid_clamped(float x) {
  if (x > 15.0f) return 1.0f;
  if (x < -15.0f) return 0.0f;
  return __fdividef(1.0f, __fadd_rn(1.0f, __expf(-x)));
}

// Three slice accumulators recombined in float32: a1 + (a2 + a3/254)/254 (two fused steps).
__device__ __forceinline__ float combine3f(uint32_t a1, uint32_t a2, uint32_t a3) {
  const float inv = 1.0f / 254.0f;
  return __fmaf_rn(__fmaf_rn((float)(int)a3, inv, (float)(int)a2), inv, (float)(int)a1);
}

// One lane of the reference's vectorised exp (internal/kernels/vec_amd64.s:282-431, the
// polynomial of FastExpF32 in vec_ops.go:104-138): clamp to [-88, 88], k = round-to-even of
// x*log2(e), r = x - k*ln2hi - k*ln2lo by fused steps, a degree-5 Taylor polynomial by fused
// Horner steps, times 2^k built from the exponent field.
__device__ __forceinline__ float ref_vec_exp(float x) {
  x = fminf(x, __int_as_float(0x42b00000));
  x = fmaxf(x, __int_as_float(0xc2b00000));
  const float k = rintf(__fmul_rn(x, __int_as_float(0x3fb8aa3b)));
  float r = __fmaf_rn(-k, __int_as_float(0x3f317200), x);
  r = __fmaf_rn(-k, __int_as_float(0x35bfbe8e), r);
  float p = __fmaf_rn(__int_as_float(0x3c088889), r, __int_as_float(0x3d2aaaab));
  p = __fmaf_rn(p, r, __int_as_float(0x3e2aaaab));
  p = __fmaf_rn(p, r, 0.5f);
  p = __fmaf_rn(p, r, 1.0f);
  p = __fmaf_rn(p, r, 1.0f);
  const int ki = (int)k + 127;
  return __fmul_rn(p, __int_as_float(ki << 23));
}

// The slice-accumulator dot product of one output, scaled like MatVecInt8 (int8.go:37-40):
// y = dot * scale (+ bias), each operation rounded.
__device__ __forceinline__ float dequant(uint32_t a1, uint32_t a2, uint32_t a3, float step, float scale) {
  const float dot = __fmul_rn(combine3f(a1, a2, a3), step);
  return __fmul_rn(dot, scale);
}

struct RowInfo {
  int session, t, pos, len;
  bool valid;
};

__device__ __forceinline__ RowInfo row_info(const BlockArgs& a, int grow) {
  RowInfo ri;
  const int tile = grow / kRows, r = grow % kRows;
  const int slot = r / a.P;
  ri.t = r % a.P;
  ri.session = tile * a.spt + slot;
  ri.valid = false;
  ri.len = 0;
  ri.pos = 0;
  if (slot < a.spt && ri.session < a.n_sess) {
    ri.len = a.seglen[ri.session];
    ri.valid = ri.t < ri.len;
    ri.pos = a.pos0[ri.session] + ri.t;
  }
  return ri;
}

}  // namespace eng
}  // namespace mc
