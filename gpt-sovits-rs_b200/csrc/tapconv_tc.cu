// tapconv_tc.cu -- bf16 tap GEMM on the 5th-generation tensor cores (tcgen05).
//
// A persistent, warp-specialised kernel.  The GEMM (gsv_internal.h) is cut
// into tiles of 128 rows (one utterance, rows q0..q0+127) x NT columns; each
// CTA walks the tiles t = blockIdx.x, blockIdx.x + gridDim.x, ... with
//   warp 0     TMA producer.  Per (segment, channel chunk) it loads ONE haloed
//              activation window [128 + span rows x CK channels] from the
//              time-major activation (3-D tensor map over (C, L, B): rows
//              outside [0, L) read as zero = the conv zero padding), into a
//              SA-deep ring; every tap of the conv is then the same window read
//              from a row-shifted shared-memory descriptor (the swizzle is a
//              function of the absolute shared address, so a K-major swizzled
//              operand may start at any row).  Weights are either resident
//              (loaded once per CTA: narrow layers) or streamed per
//              (tap, chunk) through a SB-deep ring.
//   warp 1     allocates 2 x NT TMEM columns (two accumulators) and issues
//              tcgen05.mma (M = 128, N = NT, K = 16, bf16 x bf16 -> fp32),
//              alternating accumulators between tiles so the epilogue of one
//              tile overlaps the MMAs of the next.
//   warps 2-5  epilogue: tcgen05.ld of the accumulator, bias / cond /
//              branch-average / LeakyReLU (gsv_epilogue.cuh), one 256-bit
//              bf16 store per 16-column run; then hand the accumulator back.
// A ResBlock residual enters the MMA as one more segment with identity
// weights (exact: bf16 x 1.0 accumulated in fp32), so the epilogue issues no
// global loads.  Every mbarrier wait is bounded; a wait that gives up sets
// the group's error word, stops the CTA's loops and frees its TMEM.
#include "gsv_epilogue.cuh"
#include "gsv_kernels.h"
#include "gsv_pdl.cuh"
#include "tc_common.cuh"

namespace gsv {

namespace {

constexpr int kThreads = 192;
// Segments summed over the ops of one launch (three three-piece conv2 ops of
// three segments each: small products, large product, residual).
constexpr int kMaxFlat = 9;

struct alignas(64) TcParams {
  CUtensorMap mapA[kMaxFlat];  // activation windows, one per flattened segment
  CUtensorMap mapB[kMaxFlat];  // weights [ntaps * N][Cin], one per flattened segment
  TapConvGroup grp;
  int seg_base[kMaxGroup];     // first flattened segment of each op
  int seg_minoff[kMaxFlat];    // row offset of the window start (min over taps)
  int seg_wtap0[kMaxFlat];     // resident weights: first tap tile of the segment
  int a_stage_bytes;           // bytes per A ring stage (multiple of 1024)
  int row_tiles;               // 128-row tiles per utterance (same for all ops)
  int n_tiles;                 // N / NT (same for all ops)
  int total_tiles;             // B * row_tiles * n_tiles * grp.n
  int w_tiles;                 // resident weight tiles
  int bias_off[kMaxGroup];     // each op's offset in the shared bias table
  int bias_floats;             // size of the shared bias table
  int len_smem;                // per-op valid lengths copied to shared memory (B ints each)
};

static_assert(sizeof(TcParams) <= 4096, "kernel parameter space");

// Per-op descriptor copied to shared memory at CTA start, so the roles' inner
// loops never index the kernel-parameter block dynamically.
struct SmSeg {
  int ntaps, off0, offstep, Cin, minoff, wtap0;
  short flat, pc;  // pc: piece width of three-piece operands (0: plain)
  int rows;
};
static_assert(sizeof(SmSeg) == 32, "op table layout");
struct SmOp {
  int nseg, Q, N, Cout, Lout, crop, cout_shift, bias_off;  // bias_off: into the smem bias table
  int nres, gate, bias_bc_ld, split;
  const __nv_bfloat16* res[4];
  const int* len;
  const float* bias;
  const float* bias_bc;
  __nv_bfloat16* out_raw;
  __nv_bfloat16* out_act;
  float slope, div;
  SmSeg seg[kMaxSeg];
};

static_assert(sizeof(SmOp) % 16 == 0, "16-byte aligned bias table after the op table");

// Register copy of one op's epilogue parameters for the tile being stored
// (read once per tile: loads through the shared table would be repeated after
// every global store, which may alias it).
struct EpiArgs {
  int total, N, crop, Cout, shift, lim, nres;
  const __nv_bfloat16* res[kMaxRes];  // residuals, already offset to this utterance
  const float* bias;                  // shared-memory copy of the op's bias
  const float* __restrict__ bias_bc;  // already offset to this utterance
  __nv_bfloat16* __restrict__ raw;    // already offset to this utterance
  __nv_bfloat16* __restrict__ act;
  float slope, inv_div;
  bool has_div;
  bool v8;   // both output bases 32-byte aligned: one 256-bit store per 16-column run
  bool v8r;  // every residual base 32-byte aligned: one 256-bit load per run
  bool split;  // outputs as three bf16 pieces per value ([Lout][3 Cout] rows)
};

__device__ __forceinline__ EpiArgs epi_args(const SmOp& o, const float* sbias, int b) {
  EpiArgs a;
  a.total = o.Lout * o.Cout;
  a.nres = o.nres;
#pragma unroll
  const size_t rst = (size_t)a.total * (o.split ? 3 : 1);  // elements per utterance
  for (int r = 0; r < kMaxRes; ++r)
    a.res[r] = r < o.nres ? o.res[r] + (size_t)b * rst : nullptr;
  a.N = o.N;
  a.crop = o.crop;
  a.Cout = o.Cout;
  a.shift = o.cout_shift;
  a.lim = o.len ? o.len[b] : 0x7fffffff;
  a.bias = sbias + o.bias_off;
  a.bias_bc = o.bias_bc ? o.bias_bc + (size_t)b * o.bias_bc_ld : nullptr;
  a.split = o.split != 0;
  const size_t ust = (size_t)a.total * (a.split ? 3 : 1);  // output elements per utterance
  a.raw = o.out_raw ? o.out_raw + (size_t)b * ust : nullptr;
  a.act = o.out_act ? o.out_act + (size_t)b * ust : nullptr;
  a.slope = o.slope;
  a.has_div = o.div != 1.0f;
  a.inv_div = o.div;
  a.v8 = ((reinterpret_cast<uintptr_t>(a.raw) | reinterpret_cast<uintptr_t>(a.act)) & 31) == 0;
  uintptr_t ra = 0;
#pragma unroll
  for (int r = 0; r < kMaxRes; ++r) ra |= reinterpret_cast<uintptr_t>(a.res[r]);
  a.v8r = (ra & 31) == 0;
  return a;
}

// 16 fp32 values as their three bf16 pieces at p, p + C, p + 2C: piece 0 the
// round-to-nearest bf16 of v, piece 1 that of the (exact) remainder v - piece
// 0, piece 2 that of what is left.  A normal fp32 value has 24 significant
// bits and each piece takes the next 8, so the three sum back to v exactly.
__device__ __forceinline__ void store_x3(__nv_bfloat16* p, int C, const float* v, bool v8) {
  float r[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) r[i] = v[i];
#pragma unroll
  for (int k = 0; k < 3; ++k) {
    const uint4 u0 = pack_bf16x8(r), u1 = pack_bf16x8(r + 8);
    if (k < 2) {
      const __nv_bfloat16* h0 = reinterpret_cast<const __nv_bfloat16*>(&u0);
      const __nv_bfloat16* h1 = reinterpret_cast<const __nv_bfloat16*>(&u1);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        r[i] = r[i] - __bfloat162float(h0[i]);
        r[8 + i] = r[8 + i] - __bfloat162float(h1[i]);
      }
    }
    __nv_bfloat16* q = p + (size_t)k * C;
    if (v8) {
      st_global_v8(q, u0, u1);
    } else {
      *reinterpret_cast<uint4*>(q) = u0;
      *reinterpret_cast<uint4*>(q + 8) = u1;
    }
  }
}

// Epilogue of 16 consecutive GEMM columns [n, n + 16) of row q.  Their flat
// output indices e0..e0+15 are consecutive (gsv_internal.h) and, since Cout
// and e0 are multiples of 16, lie in ONE output row t at channels c..c+15:
// one mask test, 16-byte vector bias reads from shared memory, one 256-bit
// store per output (two 16-byte ones where a base is not 32-byte aligned).
// X3: three-piece outputs and residuals (compiled only into the three-piece
// instantiations, whose register budget that code raises).
template <bool X3>
__device__ __forceinline__ void epi16(const EpiArgs& a, int q, int n, const float* acc) {
  const int e0 = q * a.N + n - a.crop;
  if (e0 < 0 || e0 >= a.total) return;  // cropped ConvTranspose rows
  const int t = a.shift >= 0 ? e0 >> a.shift : e0 / a.Cout;
  const int c = e0 - t * a.Cout;
  float v[16];
  if (t >= a.lim) {
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = 0.0f;
  } else {
    const float4* bb = reinterpret_cast<const float4*>(a.bias + c);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float4 bv = bb[k];
      v[4 * k + 0] = acc[4 * k + 0] + bv.x;
      v[4 * k + 1] = acc[4 * k + 1] + bv.y;
      v[4 * k + 2] = acc[4 * k + 2] + bv.z;
      v[4 * k + 3] = acc[4 * k + 3] + bv.w;
    }
    if (a.bias_bc != nullptr) {
      const float4* gb = reinterpret_cast<const float4*>(a.bias_bc + c);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float4 bv = __ldg(gb + k);
        v[4 * k + 0] += bv.x;
        v[4 * k + 1] += bv.y;
        v[4 * k + 2] += bv.z;
        v[4 * k + 3] += bv.w;
      }
    }
    if constexpr (X3) {  // three-piece residuals: each value the exact sum of its pieces
      const size_t at = (size_t)t * 3 * a.Cout + c;
#pragma unroll
      for (int r = 0; r < kMaxRes; ++r) {
        if (r >= a.nres) break;
        float x[16];
#pragma unroll
        for (int k = 0; k < 3; ++k) {
          const uint4* rp = reinterpret_cast<const uint4*>(a.res[r] + at + (size_t)k * a.Cout);
          uint4 ru[2];
          if (a.v8r) {
            ld_global_nc_v8(rp, ru[0], ru[1]);
          } else {
            ru[0] = __ldg(rp);
            ru[1] = __ldg(rp + 1);
          }
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&ru[h]);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const float2 f = __bfloat1622float2(h2[i]);
              x[8 * h + 2 * i] = k == 0 ? f.x : x[8 * h + 2 * i] + f.x;
              x[8 * h + 2 * i + 1] = k == 0 ? f.y : x[8 * h + 2 * i + 1] + f.y;
            }
          }
        }
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = x[i] + v[i];
      }
    }
#pragma unroll
    for (int r = 0; r < kMaxRes; ++r) {  // residual runs: 16 contiguous bf16
      if (X3 || r >= a.nres) break;
      const uint4* rp = reinterpret_cast<const uint4*>(a.res[r] + e0);
      uint4 ru[2];
      if (a.v8r) {
        ld_global_nc_v8(rp, ru[0], ru[1]);
      } else {
        ru[0] = __ldg(rp);
        ru[1] = __ldg(rp + 1);
      }
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const uint4 u = ru[k];
        const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 f = __bfloat1622float2(h2[i]);
          v[8 * k + 2 * i] = f.x + v[8 * k + 2 * i];
          v[8 * k + 2 * i + 1] = f.y + v[8 * k + 2 * i + 1];
        }
      }
    }
    if (a.has_div) {
#pragma unroll
      for (int i = 0; i < 16; ++i) v[i] = v[i] / a.inv_div;
    }
  }
  if constexpr (X3) {  // three bf16 pieces per value, planes Cout apart in the row
    const size_t at = (size_t)t * 3 * a.Cout + c;
    if (a.raw) store_x3(a.raw + at, a.Cout, v, a.v8);
    if (a.act) {
      float w[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) w[i] = lrelu(v[i], a.slope);
      store_x3(a.act + at, a.Cout, w, a.v8);
    }
    return;
  }
  const uint4 u0 = pack_bf16x8(v), u1 = pack_bf16x8(v + 8);
  // e0 is a multiple of 16 elements (32 bytes): with 32-byte aligned bases a
  // run is one full sector, written by one 256-bit store.
  if (a.raw) {
    if (a.v8) {
      st_global_v8(a.raw + e0, u0, u1);
    } else {
      *reinterpret_cast<uint4*>(a.raw + e0) = u0;
      *reinterpret_cast<uint4*>(a.raw + e0 + 8) = u1;
    }
  }
  if (a.act) {
    const __nv_bfloat162 s2 = __float2bfloat162_rn(a.slope);
    const uint4 w0 = lrelu_bf16x8(u0, s2), w1 = lrelu_bf16x8(u1, s2);
    if (a.v8) {
      st_global_v8(a.act + e0, w0, w1);
    } else {
      *reinterpret_cast<uint4*>(a.act + e0) = w0;
      *reinterpret_cast<uint4*>(a.act + e0 + 8) = w1;
    }
  }
}

template <int CK, int NT, int NBUF, int MT = 1>
struct TcShape {
  static constexpr uint32_t kBBytes = NT * CK * 2;
  static constexpr uint32_t kBPitch = (kBBytes + 1023) / 1024 * 1024;
  // Taps per streamed weight stage: one barrier wait, fence and commit per
  // stage, so narrow tiles (whose 4 MMAs per tap are short) load two taps at
  // a time.
  // (32 columns and below -- streamed only for three-piece K lists -- four.)
  static constexpr int kTapsPerB = NT <= 32 ? 4 : (NT <= 64 ? 2 : 1);
  static constexpr int kCols = NBUF * MT * NT;  // NBUF accumulators of MT x NT fp32 columns
  static constexpr uint32_t kTmemCols =
      kCols <= 32 ? 32 : (kCols <= 64 ? 64 : (kCols <= 128 ? 128 : (kCols <= 256 ? 256 : 512)));
  static_assert(kCols <= 512, "TMEM holds 512 columns");
};

// A CTA's walk over tiles t = start, start + stride, ...: tile t is the
// mixed-radix number (b, row tile, op, column tile) with the column tile
// fastest.  The stride is decomposed once; each step is digit additions with
// carries instead of three integer divisions per tile in every role.
struct TileWalker {
  int t, step, nt, oi, qt, b;
  int g_nt, g_oi, g_qt, g_b;
  int n_tiles, nops, row_tiles;
  __device__ __forceinline__ TileWalker(int start, int stride, int n_tiles_, int nops_, int row_tiles_)
      : t(start), step(stride), n_tiles(n_tiles_), nops(nops_), row_tiles(row_tiles_) {
    split(start, nt, oi, qt, b);
    split(stride, g_nt, g_oi, g_qt, g_b);
  }
  __device__ __forceinline__ void split(int x, int& a0, int& a1, int& a2, int& a3) const {
    a0 = x % n_tiles;
    x /= n_tiles;
    a1 = x % nops;
    x /= nops;
    a2 = x % row_tiles;
    a3 = x / row_tiles;
  }
  __device__ __forceinline__ void next() {
    t += step;
    nt += g_nt;
    int c = nt >= n_tiles;
    if (c) nt -= n_tiles;
    oi += g_oi + c;
    c = oi >= nops;
    if (c) oi -= nops;
    qt += g_qt + c;
    c = qt >= row_tiles;
    if (c) qt -= row_tiles;
    b += g_b + c;
  }
};

__device__ __forceinline__ bool tile_masked(const SmOp& o, int b, int q0) {
  if (o.len == nullptr) return false;
  int e = q0 * o.N - o.crop;
  if (e < 0) e = 0;
  return e / o.Cout >= o.len[b];
}

// MT: 128-row windows per tile (2: every tap issues one MMA per window into
// adjacent accumulator columns, so the per-tile hand-offs of all three roles
// are paid once per 256 rows -- the narrow layers' MMAs are too short to hide them);
// SA: activation-window ring depth (stages of MT windows); SB: streamed weight ring depth (RES = false);
// NBUF: TMEM accumulators in flight between the MMA warp and the epilogue;
// GATE: the ops are gated-activation ops (kept out of the other
// instantiations, whose register budget it would raise).
// X3: three-piece operands (K-block plane remap) and outputs.
template <int CK, int NT, bool RES, int SA, int SB, int NBUF, bool GATE, int MT, bool X3>
__global__ void __launch_bounds__(kThreads, 1) tapconv_tc_kernel(const __grid_constant__ TcParams P) {
  using S = TcShape<CK, NT, NBUF, MT>;
  static_assert(MT == 1 || ((MT == 2 || MT == 4) && !GATE), "multi-window tiles: plain epilogue only");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t a_win = (uint32_t)P.a_stage_bytes;  // one 128-row window (+ halo), 1024-aligned
  const uint32_t a_stage = MT * a_win;
  uint8_t* sA = smem;
  uint8_t* sB = smem + SA * a_stage;
  constexpr int TPB = RES ? 1 : S::kTapsPerB;
  const int nbt = RES ? P.w_tiles : SB * TPB;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sB + (size_t)nbt * S::kBPitch);
  const uint32_t a_full = smem_u32(bars);
  const uint32_t a_empty = a_full + 8 * SA;
  const uint32_t b_full = a_empty + 8 * SA;
  const uint32_t b_empty = b_full + 8 * SB;
  const uint32_t acc_full = b_empty + 8 * SB;
  const uint32_t acc_empty = acc_full + 8 * NBUF;
  const uint32_t w_full = acc_empty + 8 * NBUF;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * SA + 2 * SB + 2 * NBUF + 1);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
  SmOp* ops = reinterpret_cast<SmOp*>((reinterpret_cast<uintptr_t>(tmem_slot + 2) + 15) & ~uintptr_t(15));
  float* sbias = reinterpret_cast<float*>(ops + kMaxGroup);  // every op's bias, Cout floats each
  // Valid lengths of every op's utterances: every role tests them once per tile,
  // a dependent global load each time otherwise.
  int* slen = reinterpret_cast<int*>(sbias + P.bias_floats);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int nops = P.grp.n;
  if (threadIdx.x < nops) {
    const TapConv& g = P.grp.op[threadIdx.x];
    SmOp& o = ops[threadIdx.x];
    o.nseg = g.nseg;
    o.Q = g.Q;
    o.N = g.N;
    o.Cout = g.Cout;
    o.Lout = g.Lout;
    o.crop = g.crop;
    o.cout_shift = (g.Cout & (g.Cout - 1)) == 0 ? __ffs(g.Cout) - 1 : -1;
    o.nres = g.nres;
    o.gate = g.gate;
    o.bias_bc_ld = g.bias_bc_ld ? g.bias_bc_ld : g.Cout;
    for (int r = 0; r < kMaxRes; ++r)
      o.res[r] = r < g.nres ? static_cast<const __nv_bfloat16*>(g.res[r]) : nullptr;
    o.bias_off = P.bias_off[threadIdx.x];
    o.len = (g.len && P.len_smem) ? slen + threadIdx.x * g.B : g.len;
    o.bias = g.bias;
    o.bias_bc = g.bias_bc;
    o.out_raw = static_cast<__nv_bfloat16*>(g.out_raw);
    o.out_act = static_cast<__nv_bfloat16*>(g.out_act);
    o.slope = g.slope;
    o.div = g.div;
    o.split = g.split;
    for (int s = 0; s < g.nseg; ++s) {
      const int f = P.seg_base[threadIdx.x] + s;
      SmSeg& d = o.seg[s];
      d.ntaps = g.seg[s].ntaps;
      d.off0 = g.seg[s].off0;
      d.offstep = g.seg[s].offstep;
      d.Cin = g.seg[s].Cin;
      d.minoff = P.seg_minoff[f];
      d.wtap0 = P.seg_wtap0[f];
      d.pc = (short)g.seg[s].pc;
      d.flat = (short)f;
      d.rows = kM + (d.ntaps - 1) * abs(d.offstep);
    }
  }
  for (int o = 0; o < nops; ++o)
    for (int c = threadIdx.x; c < P.grp.op[o].Cout; c += kThreads)
      sbias[P.bias_off[o] + c] = P.grp.op[o].bias[c];
  if (threadIdx.x == 0) {
    for (int s = 0; s < SA; ++s) {
      mbar_init(a_full + 8 * s, 1);
      mbar_init(a_empty + 8 * s, 1);
    }
    for (int s = 0; s < SB; ++s) {
      mbar_init(b_full + 8 * s, 1);
      mbar_init(b_empty + 8 * s, 1);
    }
    for (int s = 0; s < NBUF; ++s) {
      mbar_init(acc_full + 8 * s, 1);
      mbar_init(acc_empty + 8 * s, 4);
    }
    mbar_init(w_full, 1);
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) tmem_alloc(smem_u32(tmem_slot), S::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // Everything above touched only this CTA's resources, the kernel parameters
  // and the static biases; activations and lengths come from earlier kernels.
  pdl_wait();
  if (P.len_smem) {
    for (int o = 0; o < nops; ++o)
      if (P.grp.op[o].len)
        for (int b = threadIdx.x; b < P.grp.op[o].B; b += kThreads) slen[o * P.grp.op[o].B + b] = P.grp.op[o].len[b];
    __syncthreads();
  }
  const uint32_t tmem = *tmem_slot;
  int* err = P.grp.err;
  const int row_tiles = MT == 1 ? P.row_tiles : cdiv(P.row_tiles, MT), n_tiles = P.n_tiles;
  const int total = P.total_tiles / P.row_tiles * row_tiles;
  constexpr int kTileRows = kM * MT;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      bool ok = true;
      if (RES) {
        mbar_expect_tx(w_full, (uint32_t)P.w_tiles * S::kBBytes);
        // Tile (chunk c0 / CK, tap j) of a segment at wtap0 + (c0 / CK) * ntaps + j.
        for (int o = 0; o < nops; ++o)
          for (int s = 0; s < ops[o].nseg; ++s) {
            const SmSeg& d = ops[o].seg[s];
            for (int c0 = 0; c0 < d.Cin; c0 += CK)
              for (int j = 0; j < d.ntaps; ++j)
                tma_load_2d(smem_u32(sB + (size_t)(d.wtap0 + (c0 / CK) * d.ntaps + j) * S::kBPitch),
                            &P.mapB[d.flat], w_full, c0, j * ops[o].N);
          }
      }
      for (int o = 0; o < nops; ++o)
        for (int s = 0; s < ops[o].nseg; ++s) {
          const int f = ops[o].seg[s].flat;
          asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&P.mapA[f])) : "memory");
          if (!RES)
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&P.mapB[f])) : "memory");
        }
      uint32_t ia = 0, ib = 0;
      for (TileWalker w(blockIdx.x, gridDim.x, n_tiles, nops, row_tiles); w.t < total && ok; w.next()) {
        const int oi = w.oi, n0 = w.nt * NT, b = w.b, q0 = w.qt * kTileRows;
        if (tile_masked(ops[oi], b, q0)) continue;
        const int nseg = ops[oi].nseg, N = ops[oi].N;
        for (int s = 0; s < nseg && ok; ++s) {
          const SmSeg d = ops[oi].seg[s];  // register copy (the asm below clobbers memory)
          const uint32_t wbytes = (uint32_t)d.rows * CK * 2;
          for (int c0 = 0; c0 < d.Cin && ok; c0 += CK) {
            const uint32_t st = ia % SA;
            if (!mbar_wait(a_empty + 8 * st, ((ia / SA) & 1u) ^ 1u, abort)) {
              raise_err(err, abort, 1);
              ok = false;
              break;
            }
            mbar_expect_tx(a_full + 8 * st, MT * wbytes);
            // Three-piece operands: K block c0 / pc of the five-block list reads
            // plane 2, 1, 0, 1, 0, of the three-block list (a residual against
            // identities) 2, 1, 0, the one-block list plane 0.
            int ac0 = c0;
            if (X3 && d.pc) {
              const int kb = c0 / d.pc, r = c0 - kb * d.pc;
              const int plane = d.Cin == d.pc ? 0 : (kb == 0 ? 2 : (kb & 1 ? 1 : 0));
              ac0 = plane * d.pc + r;
            }
#pragma unroll
            for (int m = 0; m < MT; ++m)
              tma_load_3d(smem_u32(sA + st * a_stage + m * a_win), &P.mapA[d.flat], a_full + 8 * st, ac0,
                          q0 + m * kM + d.minoff, b);
            ++ia;
            if (!RES) {
              for (int j = 0; j < d.ntaps; j += TPB) {
                const int nt = min(TPB, d.ntaps - j);
                const uint32_t sb = ib % SB;
                if (!mbar_wait(b_empty + 8 * sb, ((ib / SB) & 1u) ^ 1u, abort)) {
                  raise_err(err, abort, 2);
                  ok = false;
                  break;
                }
                mbar_expect_tx(b_full + 8 * sb, (uint32_t)nt * S::kBBytes);
                for (int t = 0; t < nt; ++t)
                  tma_load_2d(smem_u32(sB + (sb * TPB + t) * S::kBPitch), &P.mapB[d.flat], b_full + 8 * sb,
                              c0, (j + t) * N + n0);
                ++ib;
              }
            }
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16<NT>();
      bool ok = true;
      if (RES && !mbar_wait(w_full, 0, abort)) {
        raise_err(err, abort, 3);
        ok = false;
      }
      uint32_t ia = 0, ib = 0, i = 0;
      for (TileWalker w(blockIdx.x, gridDim.x, n_tiles, nops, row_tiles); w.t < total && ok; w.next(), ++i) {
        const int oi = w.oi, b = w.b, q0 = w.qt * kTileRows;
        const bool masked = tile_masked(ops[oi], b, q0);
        const int nseg = ops[oi].nseg;
        const uint32_t buf = i % NBUF;
        if (!mbar_wait_fast(acc_empty + 8 * buf, ((i / NBUF) & 1u) ^ 1u, abort)) {
          raise_err(err, abort, 4);
          break;
        }
        tc_fence_after();
        if (masked) {
          mbar_arrive(acc_full + 8 * buf);
          continue;
        }
        const uint32_t d = tmem + buf * (MT * NT);
        // The single issuing thread is the pace-setter of narrow tiles (a
        // measured 45-64 cycles per MMA when the issue loop is straight-line
        // code, several times that with per-MMA address and descriptor
        // arithmetic): descriptors are built once per window / weight stage
        // and advanced by constant adds (the 14-bit start-address field of a
        // descriptor holds address >> 4, so byte offsets that keep the operand
        // inside shared memory add as offset >> 4), and the first MMA of each
        // window, which starts the accumulator, is issued on its own.
        bool first = true;
        constexpr uint64_t kK = 2;  // one 16-element K step = 32 bytes along the row
        const uint64_t win_d = (uint64_t)(a_win >> 4);
        for (int s = 0; s < nseg && ok; ++s) {
          const SmSeg sg = ops[oi].seg[s];  // register copy
          for (int c0 = 0; c0 < sg.Cin && ok; c0 += CK) {
            const uint32_t st = ia % SA;
            if (!mbar_wait_fast(a_full + 8 * st, (ia / SA) & 1u, abort)) {
              raise_err(err, abort, 5);
              ok = false;
              break;
            }
            tc_fence_after();
            uint64_t ad = sdesc<CK>(smem_u32(sA + st * a_stage) + (uint32_t)(sg.off0 - sg.minoff) * (CK * 2));
            const uint64_t ad_step = (uint64_t)(int64_t)(sg.offstep * (CK * 2 / 16));  // one tap: offstep rows
            // All K steps of one tap: window row shift in `ad`, weights in `bt`.
            auto tap_mmas = [&](uint64_t bt) {
#pragma unroll
              for (int kk = 0; kk < CK / 16; ++kk) {
#pragma unroll
                for (int m = 0; m < MT; ++m) {
                  if (kk == 0 && first)
                    mma_bf16_first(d + m * NT, ad + m * win_d, bt, idesc);
                  else
                    mma_bf16_acc(d + m * NT, ad + m * win_d + kk * kK, bt + kk * kK, idesc);
                }
                first = false;
              }
              ad += ad_step;
            };
            if (RES) {
              uint64_t bd = sdesc<CK>(smem_u32(sB + (size_t)(sg.wtap0 + (c0 / CK) * sg.ntaps) * S::kBPitch));
#pragma unroll 2
              for (int j = 0; j < sg.ntaps; ++j) {
                tap_mmas(bd);
                bd += S::kBPitch >> 4;
              }
            } else {
              for (int j = 0; j < sg.ntaps; j += TPB) {
                const uint32_t sb = ib % SB;
                if (!mbar_wait_fast(b_full + 8 * sb, (ib / SB) & 1u, abort)) {
                  raise_err(err, abort, 6);
                  ok = false;
                  break;
                }
                tc_fence_after();
                const uint64_t bd = sdesc<CK>(smem_u32(sB + sb * TPB * S::kBPitch));
#pragma unroll
                for (int t = 0; t < TPB; ++t)
                  if (t == 0 || j + t < sg.ntaps) tap_mmas(bd + (uint64_t)t * (S::kBPitch >> 4));
                mma_commit(b_empty + 8 * sb);
                ++ib;
              }
            }
            mma_commit(a_empty + 8 * st);
            ++ia;
          }
        }
        mma_commit(acc_full + 8 * buf);  // arrives once this tile's MMAs complete
      }
    }
  } else {
    // ----------------------------------------------------------- epilogue
    const int quarter = warp & 3;  // TMEM lanes this warp may access
    const int row = quarter * 32 + lane;
    const uint32_t lane_addr = tmem + ((uint32_t)(quarter * 32) << 16);
    uint32_t i = 0;
    for (TileWalker w(blockIdx.x, gridDim.x, n_tiles, nops, row_tiles); w.t < total; w.next(), ++i) {
      const int oi = w.oi, n0 = w.nt * NT, b = w.b;
      const SmOp& o = ops[oi];
      const uint32_t buf = i % NBUF;
      const bool ok = mbar_wait_fast(acc_full + 8 * buf, (i / NBUF) & 1u, abort);
      if (!__all_sync(0xffffffffu, ok)) {
        if (lane == 0) raise_err(err, abort, 7);
        break;
      }
      tc_fence_after();
      const EpiArgs ea = epi_args(o, sbias, b);
#pragma unroll 1
      for (int m = 0; m < MT; ++m) {
        const int q0 = w.qt * kTileRows + m * kM;
        const uint32_t acc = lane_addr + buf * (MT * NT) + m * NT;  // this window's accumulator
        const bool masked = tile_masked(o, b, q0);
        const int q = q0 + row;
        const bool live = q < o.Q;
        if (GATE) {
          // Gated activation: 32-column runs (a | b) -> 16 outputs of channel
          // block (n0 + c0) / 2 (WN, src/models/sovits_flow.rs:171-184).
          const int H = o.Cout / 2;
          const bool dead = q >= ea.lim || q >= o.Q;
#pragma unroll 1
          for (int c0 = 0; c0 < NT; c0 += 32) {
            float va[16], vb[16];
            if (!masked) {
              tmem_ld16(acc + (uint32_t)c0, va);
              tmem_ld16(acc + (uint32_t)(c0 + 16), vb);
            }
            if (!live) continue;
            const int n = n0 + c0;
            float y[16];
#pragma unroll
            for (int k = 0; k < 16; ++k) {
              float a = va[k] + ea.bias[n + k], sg = vb[k] + ea.bias[n + 16 + k];
              if (ea.bias_bc) {
                a = a + __ldg(ea.bias_bc + n + k);
                sg = sg + __ldg(ea.bias_bc + n + 16 + k);
              }
              y[k] = (masked || dead) ? 0.0f : tanhf(a) * (1.0f / (1.0f + expf(-sg)));
            }
            __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(o.out_raw) + ((size_t)b * o.Lout + q) * H + n / 2;
            if (ea.v8) {  // 16 outputs = 32 bytes at a 16-channel offset (H % 16 == 0)
              st_global_v8(dst, pack_bf16x8(y), pack_bf16x8(y + 8));
            } else {
              store8(dst, y);
              store8(dst + 8, y + 8);
            }
          }
          continue;
        }
#pragma unroll 1
        for (int c0 = 0; c0 < NT; c0 += 16) {
          float v[16];
          if (!masked) {
            tmem_ld16(acc + (uint32_t)c0, v);
          } else {
#pragma unroll
            for (int k = 0; k < 16; ++k) v[k] = 0.0f;
          }
          if (live) epi16<X3>(ea, q, n0 + c0, v);
        }
      }  // windows of the tile
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acc_empty + 8 * buf);
    }
  }
  // This CTA's work is done: the next kernel's CTAs may be scheduled.
  pdl_trigger();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, S::kTmemCols);
  }
}

// ------------------------------------------------------------------- host side
template <int CK, int NT, bool RES, int SA, int SB, int NBUF, int MT = 1>
size_t cfg_smem(const TcParams& P) {
  using S = TcShape<CK, NT, NBUF, MT>;
  const int nbt = RES ? P.w_tiles : SB * S::kTapsPerB;
  return 1024 + (size_t)SA * MT * P.a_stage_bytes + (size_t)nbt * S::kBPitch +
         8 * (2 * SA + 2 * SB + 2 * NBUF + 1) + 32 + sizeof(SmOp) * kMaxGroup +
         sizeof(float) * (size_t)P.bias_floats +
         (P.len_smem ? sizeof(int) * (size_t)kMaxGroup * P.grp.op[0].B : 0);
}

// True when `per_sm` CTAs of this configuration fit one SM's shared memory.
template <int CK, int NT, bool RES, int SA, int SB, int NBUF, int MT = 1>
bool cfg_fits(const TcParams& P, int per_sm) {
  return per_sm * (cfg_smem<CK, NT, RES, SA, SB, NBUF, MT>(P) + 1024) <= (size_t)smem_per_sm();
}

template <int CK, int NT, bool RES, int SA, int SB, int NBUF, bool GATE = false, int MT = 1, bool X3 = false>
cudaError_t launch_cfg(TcParams& P, cudaStream_t st) {
  using S = TcShape<CK, NT, NBUF, MT>;
  const size_t smem = cfg_smem<CK, NT, RES, SA, SB, NBUF, MT>(P);
  if (smem > 227 * 1024) return cudaErrorInvalidValue;
  auto kern = tapconv_tc_kernel<CK, NT, RES, SA, SB, NBUF, GATE, MT, X3>;
  // CTAs per SM, bounded by shared memory (1 KB reserved per CTA), registers,
  // threads and TMEM (each CTA holds kTmemCols of the SM's 512 columns).
  int nregs = 0;
  cudaError_t e = kernel_setup(kern, smem, &nregs);
  if (e != cudaSuccess) return e;
  const int smem_sm = smem_per_sm();
  const int regs_cta = ((nregs * 32 + 255) / 256 * 256) * (kThreads / 32);
  int per_sm = std::min({smem_sm / (int)(smem + 1024), 65536 / std::max(regs_cta, 1),
                         2048 / kThreads, (int)(512 / S::kTmemCols)});
  per_sm = std::max(1, per_sm);
  const int tiles = P.total_tiles / P.row_tiles * cdiv(P.row_tiles, MT);
  const int grid = std::min(tiles, sm_count() * per_sm);
  if (grid <= 0) return cudaSuccess;
  const size_t smem_launch = pad_smem_to_occupancy(smem, per_sm, smem_sm);
  e = kernel_setup(kern, smem_launch, &nregs);
  if (e != cudaSuccess) return e;
  {
    const cudaError_t e_ = launch_k(kern, grid, kThreads, smem_launch, st, P);
    if (e_ != cudaSuccess) return e_;
  }
  return cudaGetLastError();
}

}  // namespace

// Configurations of the three-piece ops (GSV_MODE_FP32_TC), instantiated
// apart from the bf16 ones so that the bf16 kernels keep their register budget.
// Narrow layers (whose K lists span several channel chunks) keep every chunk's
// weights resident where that fits one CTA per SM, else stream four taps per
// stage over two-window tiles; wider ones take the bf16 choices.
static cudaError_t launch_x3(TcParams& P, int ck, int nt, bool spare, bool branch_sum, cudaStream_t st) {
  if (ck == 16 && nt == 16 && P.n_tiles == 1) {
    if (spare && cfg_fits<16, 16, true, 3, 1, 4, 4>(P, 1)) return launch_cfg<16, 16, true, 3, 1, 4, false, 4, true>(P, st);
    if (cfg_fits<16, 16, true, 4, 1, 4>(P, 1)) return launch_cfg<16, 16, true, 4, 1, 4, false, 1, true>(P, st);
    return launch_cfg<16, 16, false, 2, 4, 4, false, 2, true>(P, st);
  }
  if (ck == 32 && nt == 32 && P.n_tiles == 1) {
    if (spare && cfg_fits<32, 32, true, 2, 1, 4, 2>(P, 1)) return launch_cfg<32, 32, true, 2, 1, 4, false, 2, true>(P, st);
    if (cfg_fits<32, 32, true, 3, 1, 4>(P, 1)) return launch_cfg<32, 32, true, 3, 1, 4, false, 1, true>(P, st);
    return launch_cfg<32, 32, false, 2, 4, 4, false, 2, true>(P, st);
  }
  if (ck == 64 && nt == 256) return launch_cfg<64, 256, false, 3, 4, 2, false, 1, true>(P, st);
  if (ck == 64 && nt == 128) return launch_cfg<64, 128, false, 2, 3, 2, false, 1, true>(P, st);
  if (ck == 64 && nt == 64) {
    if (branch_sum) return spare ? launch_cfg<64, 64, false, 2, 2, 2, false, 2, true>(P, st)
                                 : launch_cfg<64, 64, false, 3, 2, 4, false, 1, true>(P, st);
    if (spare && cfg_fits<64, 64, false, 2, 2, 2, 2>(P, 2)) return launch_cfg<64, 64, false, 2, 2, 2, false, 2, true>(P, st);
    return cfg_fits<64, 64, false, 2, 4, 4>(P, 2) ? launch_cfg<64, 64, false, 2, 4, 4, false, 1, true>(P, st)
                                                 : launch_cfg<64, 64, false, 3, 2, 4, false, 1, true>(P, st);
  }
  return cudaErrorInvalidValue;
}

// Channel width that sets a segment's chunk: its piece width for three-piece
// operands, else its input width.
static int seg_width(const TapSeg& s) { return s.pc ? s.pc : s.Cin; }

bool tapconv_tc_supported(const TapConv& op) {
  if (op.nseg < 1 || op.nseg > kMaxSeg) return false;
  const int cin = op.seg[0].Cin, cw = seg_width(op.seg[0]);
  for (int s = 0; s < op.nseg; ++s) {
    const TapSeg& sg = op.seg[s];
    if (sg.ntaps < 1) return false;
    if ((sg.ntaps - 1) * abs(sg.offstep) > 256 - kM) return false;  // TMA box rows
    if (sg.pc) {  // a K list over three pieces: every segment the same piece width
      if (sg.pc != cw || sg.pc > 4096 || (sg.Cin != sg.pc && sg.Cin != 3 * sg.pc && sg.Cin != 5 * sg.pc))
        return false;
    } else if (sg.Cin != cin || op.seg[0].pc) {
      return false;
    }
  }
  if (op.split && (op.gate || !op.seg[0].pc)) return false;
  const int ck = ck_for(cw), nt = nt_for(op.N);
  if (!ck || !nt || op.N % nt) return false;
  if (op.Cout % 16) return false;  // 16-element epilogue runs stay 32-byte aligned
  if (op.gate && (op.N != op.Cout || op.N % 32 || op.crop || op.Q != op.Lout || op.nres)) return false;
  if ((long long)op.Lout * op.Cout >= (1ll << 31) || (long long)op.Q * op.N >= (1ll << 31))
    return false;  // 32-bit per-utterance index math
  return (ck == 64 && (nt == 256 || nt == 128 || nt == 64)) || (ck == 32 && nt == 32) ||
         (ck == 16 && nt == 16);
}

cudaError_t launch_tapconv_tc(const TapConvGroup& g, cudaStream_t st) {
  if (!encode_fn()) return cudaErrorNotSupported;
  if (g.n < 1 || g.n > kMaxGroup) return cudaErrorInvalidValue;
  TcParams P;
  memset(&P, 0, sizeof P);
  P.grp = g;
  const int ck = ck_for(seg_width(g.op[0].seg[0]));
  int nt = nt_for(g.op[0].N);
  // A launch that would not fill the SMs (a short utterance, one time chunk
  // of a long one) runs each tile's whole MMA chain on its own: narrower
  // column tiles halve that chain and double the tiles.  Each output column's
  // arithmetic is the same, so are the samples.
  bool gated = false;
  for (int i = 0; i < g.n; ++i) gated = gated || g.op[i].gate;
  if (ck == 64 && !gated) {
    long long tiles = (long long)g.op[0].B * cdiv(g.op[0].Q, kM) * (g.op[0].N / std::max(nt, 1)) * g.n;
    while (nt > 64 && tiles < sm_count() && g.op[0].N % (nt / 2) == 0) {
      nt /= 2;
      tiles *= 2;
    }
  }
  int nflat = 0, wtiles = 0, max_rows = 0;
  for (int i = 0; i < g.n; ++i) {
    TapConv& op = P.grp.op[i];
    if (!tapconv_tc_supported(op) || ck_for(seg_width(op.seg[0])) != ck || op.N % nt ||
        op.N != g.op[0].N || op.Q != g.op[0].Q || op.B != g.op[0].B)
      return cudaErrorInvalidValue;
    op.row_tiles = cdiv(op.Q, kM);
    P.seg_base[i] = nflat;
    for (int s = 0; s < op.nseg; ++s, ++nflat) {
      if (nflat >= kMaxFlat) return cudaErrorInvalidValue;
      const TapSeg& sg = op.seg[s];
      const int rows = window_rows(sg);
      max_rows = std::max(max_rows, rows);
      P.seg_minoff[nflat] = sg.offstep >= 0 ? sg.off0 : sg.off0 + (sg.ntaps - 1) * sg.offstep;
      P.seg_wtap0[nflat] = wtiles;
      wtiles += sg.ntaps * (sg.Cin / ck);
      if (!encode_act(&P.mapA[nflat], sg.x, op.B, sg.Lin, sg.pc ? 3 * sg.pc : sg.Cin, ck, rows))
        return cudaErrorInvalidValue;
      if (!encode_w(&P.mapB[nflat], sg.w, sg.ntaps * op.N, sg.Cin, ck, nt)) return cudaErrorInvalidValue;
    }
  }
  int boff = 0;
  for (int i = 0; i < g.n; ++i) {
    P.bias_off[i] = boff;
    boff += g.op[i].Cout;
  }
  P.bias_floats = boff;
  P.len_smem = g.op[0].B <= 1024;
  P.row_tiles = P.grp.op[0].row_tiles;
  P.n_tiles = g.op[0].N / nt;
  P.total_tiles = g.op[0].B * P.row_tiles * P.n_tiles * g.n;
  P.a_stage_bytes = (max_rows * ck * 2 + 1023) / 1024 * 1024;
  P.w_tiles = wtiles;
  if (P.total_tiles <= 0) return cudaSuccess;
  bool gate = false;
  for (int i = 0; i < g.n; ++i) gate = gate || g.op[i].gate;
  // The three-branch sum (one GEMM over the branches' last convs, plus their
  // residuals as identity segments at >= 32 channels) has >= 3 segments.
  bool branch_sum = false;
  for (int i = 0; i < g.n; ++i) branch_sum = branch_sum || g.op[i].nseg >= 3;
  if (gate) {
    for (int i = 0; i < g.n; ++i)
      if (!g.op[i].gate) return cudaErrorInvalidValue;  // a group is all gated or none
    if (ck == 64 && nt == 128) return launch_cfg<64, 128, false, 2, 3, 2, true>(P, st);
    return cudaErrorNotSupported;
  }
  // Narrow layers keep every weight tile of the launch resident in shared
  // memory.  Multi-window tiles (MT = 2, 4) divide the per-tile hand-offs
  // where those bound the launch (measured per op kind on B200): four windows
  // for the 16-channel convs (rb4 step-2 conv1 0.336 -> 0.274 ms against two),
  // two for the 32-channel ones, every narrow op except the 16-channel branch
  // sum, which is bound by its epilogue and keeps one window with more CTAs
  // per SM; at 64 channels the branch sum, whose long MMA chains outweigh the
  // lost second CTA per SM, and the convs where two CTAs still fit.  Every
  // epilogue writes with 256-bit stores: they beat the shared-memory staged
  // TMA-store epilogue this kernel used to have for two-output layers (conv2
  // 3-9 % at 64-256 channels, the stride-2 ConvTranspose 10 %).
  // Multi-window tiles only where the launch has tiles to spare: they divide
  // the tile count, and a sub-wave launch is bound by one tile's chain.
  const bool spare = P.total_tiles >= 4 * sm_count();
  bool x3 = false, multi = false, sum3 = false;
  for (int i = 0; i < g.n; ++i) {
    x3 = x3 || g.op[i].split;
    sum3 = sum3 || g.op[i].nres >= 2;
    for (int s = 0; s < g.op[i].nseg; ++s) multi = multi || g.op[i].seg[s].Cin > ck;
  }
  if (x3) {
    for (int i = 0; i < g.n; ++i)
      if (!g.op[i].split) return cudaErrorInvalidValue;  // a group is all three-piece or none
    return launch_x3(P, ck, nt, spare, sum3, st);
  }
  // The resident-weight configurations below hold one channel chunk per tap.
  if (multi && ck < 64) return cudaErrorInvalidValue;
  if (ck == 16 && nt == 16 && P.n_tiles == 1) {
    if (branch_sum || !spare) return launch_cfg<16, 16, true, 6, 1, 4>(P, st);
    return launch_cfg<16, 16, true, 3, 1, 4, false, 4>(P, st);
  }
  if (ck == 32 && nt == 32 && P.n_tiles == 1)
    return spare ? (branch_sum ? launch_cfg<32, 32, true, 3, 1, 4, false, 2>(P, st)
                               : launch_cfg<32, 32, true, 2, 1, 4, false, 2>(P, st))
                 : launch_cfg<32, 32, true, 3, 1, 4>(P, st);
  // 256 columns (one CTA per SM): three window stages (rb0 conv2 / branch sum
  // 2-6 % faster than two).
  if (ck == 64 && nt == 256) return launch_cfg<64, 256, false, 3, 4, 2>(P, st);
  if (ck == 64 && nt == 128) return launch_cfg<64, 128, false, 2, 3, 2>(P, st);
  if (ck == 64 && nt == 64) {
    if (branch_sum) return spare ? launch_cfg<64, 64, false, 2, 2, 2, false, 2>(P, st)
                                 : launch_cfg<64, 64, false, 3, 2, 4>(P, st);
    // Two-window tiles (one weight stage serves 256 rows) where two CTAs per
    // SM still fit (measured on B200: the dilation-1 conv1 0.321 -> 0.297 ms),
    // else -- the wider windows of dilations 3 / 5 -- with a single window
    // stage, the other CTA on the SM covering the next window's load (0.33 /
    // 0.35 -> 0.30 ms, forward -1 % sustained).
    if (spare && cfg_fits<64, 64, false, 2, 2, 2, 2>(P, 2)) return launch_cfg<64, 64, false, 2, 2, 2, false, 2>(P, st);
    if (spare && cfg_fits<64, 64, false, 1, 3, 2, 2>(P, 2)) return launch_cfg<64, 64, false, 1, 3, 2, false, 2>(P, st);
    // Else four weight stages (eight taps in flight) where that still fits
    // two CTAs per SM: the 64-column MMAs are short, and with two stages the
    // MMA warp waited on weight loads (4-8 % faster).
    return cfg_fits<64, 64, false, 2, 4, 4>(P, 2) ? launch_cfg<64, 64, false, 2, 4, 4>(P, st)
                                                 : launch_cfg<64, 64, false, 3, 2, 4>(P, st);
  }
  return cudaErrorInvalidValue;
}

}  // namespace gsv
