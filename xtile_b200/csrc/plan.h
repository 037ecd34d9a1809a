// Mapping of one xt Block program onto a B200 kernel family.
//
// The reference lowers a program by unrolling its grid (xt-serialize) and
// rewriting every tile op into NPU commands (xt-to-nova, nova-*).  Here the
// Block program is classified once; the grid becomes the CUDA launch and the
// tile ops become one of four sm_100a kernels:
//
//   ew     flat elementwise map (add/sub/mul/unary/casts) over whole arrays
//   rows   row programs: loads of full rows, elementwise + row reductions +
//          row broadcasts (the softmax chain), one warp per row
//   gemm   matmul / K-looped matmul-add chains / mma with a fused epilogue of
//          row or scalar scale and bias and an optional int8 cast
//          (tcgen05 + TMEM + TMA)
//   conv   load_conv2d as an implicit GEMM (tcgen05 + TMEM + TMA)
//   tile   any other Block program (reshape / transpose / permute,
//          reductions along any axis, broadcasting binaries, tensor
//          constants): one CTA per Block interprets the tile ops on f32 tiles
//          held in shared memory
#pragma once

#include <cstdint>
#include <string>
#include <vector>

#include "ir.h"

namespace xt {

enum class Family { Ew = 1, Rows = 2, Gemm = 3, Conv = 4, Tile = 5 };

// --- elementwise --------------------------------------------------------------
// Register programs shared by the ew and rows kernels.  ``dst``/``a``/``b``
// index value registers; Load reads input slot ``a``; Store writes register
// ``a`` to output slot ``dst``.
enum Opcode : uint8_t {
  kLoad = 1, kStore, kAdd, kSub, kMul, kExp, kCos, kSin, kRecip, kRsqrt, kSigmoid, kTanh,
  kSilu, kItof, kFtoi,
  // rows-only: a row register holds one full row; a scalar register one value
  // per row.  ``kBcast*`` take a row (a) and a scalar (b).
  kBcastAdd, kBcastSub, kBcastMul, kRowMax, kRowSum, kLoadScalar, kStoreScalar,
};

struct Instr {
  uint8_t op, dst, a, b;
};

constexpr int kMaxInstr = 48;
constexpr int kMaxSlots = 6;

struct EwPlan {
  int n_in = 0, n_out = 0;
  int in_arg[kMaxSlots], out_arg[kMaxSlots];
  Elem in_elem[kMaxSlots], out_elem[kMaxSlots];
  std::vector<Instr> code;
  int n_regs = 0;
  int64_t numel = 0;            // elements of each (identically shaped) array
  int64_t bid0_span = 0;        // elements covered by one bid0 step (0: bid0 unused)
  std::vector<int64_t> shape;
  // inputs that are a [1, C] row broadcast over the [R, C] arrays: element i
  // of the flat map reads element i mod C of the row (bcast_period = C)
  bool in_bcast[kMaxSlots] = {};
  int64_t bcast_period = 0;
};

struct RowPlan {
  int n_in = 0, n_out = 0;
  int in_arg[kMaxSlots], out_arg[kMaxSlots];
  bool in_is_scalar[kMaxSlots], out_is_scalar[kMaxSlots];
  std::vector<Instr> code;
  int n_vregs = 0, n_sregs = 0;
  int64_t rows = 0, cols = 0;   // covered rows; full row length
  int64_t tile_rows = 0;        // rows per Block (bid0 step)
  int row_axis = 0;             // bid axis indexing the rows
  bool softmax = false;         // the max/sub/exp/sum/reciprocal/mul chain
};

// --- gemm ---------------------------------------------------------------------
enum EpiKind : uint8_t { kEpiMulRow = 1, kEpiAddRow, kEpiMulScalar, kEpiAddScalar };
struct EpiStep {
  uint8_t kind;
  int arg;
};

struct GemmPlan {
  int a_arg = -1, b_arg = -1, c_arg = -1, acc_arg = -1;  // acc_arg: xt.mma accumulator input
  Elem ab_elem = Elem::Unknown, c_elem = Elem::F32;
  int64_t M = 0, N = 0, K = 0;       // covered extents
  int64_t lda = 0, ldb = 0, ldc = 0;  // row strides in elements
  int64_t tm = 0, tn = 0, tk = 0;    // Block tile of the program
  int k_steps = 1;                    // matmul terms summed along K
  int m_axis = 0, n_axis = 1;         // bid axes selecting the M / N tile
  std::vector<EpiStep> epi;
  bool ftoi = false;
};

// --- conv -----------------------------------------------------------------------
struct ConvPlan {
  int in_arg = -1, filt_arg = -1, out_arg = -1;
  Elem elem = Elem::Unknown;
  int64_t N = 0, H = 0, W = 0, C = 0;        // input NHWC
  int64_t KH = 0, KW = 0, KO = 0;            // filter HWIO (KO = filter output channels)
  int64_t ON = 0, OH = 0, OW = 0, OC = 0;    // covered output extents
  int64_t out_h = 0, out_w = 0, out_c = 0;   // output array dims (row strides)
  int64_t pad_t = 0, pad_l = 0, stride_h = 1, stride_w = 1, dil_h = 1, dil_w = 1;
  int64_t tb = 1, th = 0, tw = 0;            // Block tile
  int n_axis = 0;                            // bid axis of the batch tile
};

// Whether a row program runs the generated one-warp-per-row kernel: rows of
// at most 2048 columns whose ``n_v`` live rows a lane holds in at most 160
// values (float4 groups, or elements when the rows are not whole groups).
inline bool row_warp_fits(int64_t cols, int n_v) {
  return cols <= 2048 && n_v * 4 * (((cols + 3) / 4 + 31) / 32) <= 160 && n_v * ((cols + 31) / 32) <= 160;
}

// Threads per row of the generated one-CTA-per-row kernel for rows of
// ``cols`` columns with ``n_v`` live rows: the fewest (128 to 1024, powers of
// two) with which a thread holds at most 8 four-element groups (or 32
// elements) of each live row; 0 when no CTA holds them.  The planner takes a
// row program only when this is not 0.
inline int row_cta_threads(int64_t cols, int n_v) {
  for (int t = 128; t <= 1024; t *= 2)
    if (n_v * ((cols + 4 * t - 1) / (4 * t)) <= 8 && n_v * ((cols + t - 1) / t) <= 32) return t;
  return 0;
}

// --- tile -----------------------------------------------------------------------
// Shapes are padded with leading 1s to rank 4 (tile and array rank agree).
enum TileOpKind : uint8_t {
  kTLoad = 1, kTStore, kTConst, kTUnary, kTBinary, kTReduce, kTReshape, kTPermute,
};
constexpr int kTileRank = 4;
constexpr int kTileMaxVals = 16;
constexpr int kTileMaxOps = 32;
constexpr int kTileMaxArgs = 8;
constexpr int kTileSmemFloats = 48 * 1024;  // 192 KiB of shared memory per Block

struct TileVal {               // one tile value, f32 elements in shared memory
  int32_t shape[kTileRank];
  int32_t stride[kTileRank];   // shared-memory strides in floats (rows padded to an odd length)
  int32_t offset;              // first float
  int32_t numel;
  uint8_t i8;                  // int8 value: add/sub/mul results wrap modulo 256
};

struct TileOp {
  uint8_t kind;                // TileOpKind
  uint8_t code;                // unary / binary: Opcode (kExp.., kAdd.., kItof, kFtoi); reduce: 0 max, 1 sum;
                               // store: 1 = value ``a`` is permute(``b``, perm), read from ``b`` (``a`` has no slot data)
  uint8_t dst, a, b;           // value indices (store: ``a`` is the stored value)
  uint8_t arg;                 // load / store: argument slot
  uint8_t axis;                // reduce: the reduced dim
  uint8_t perm[kTileRank];     // permute (and store code 1): dst dim d is src dim perm[d]
  int8_t coord_bid[kTileRank]; // load / store tile coordinate per dim: bid axis, or -1 for ``coord``
  int32_t coord[kTileRank];
  float value;                 // constant splat
};

struct TilePlan {
  int n_args = 0;
  int arg[kTileMaxArgs];                 // function argument of each slot
  Elem arg_elem[kTileMaxArgs];
  int32_t arg_shape[kTileMaxArgs][kTileRank];
  std::vector<TileVal> vals;
  std::vector<TileOp> ops;
  int32_t smem_floats = 0;
};

struct Plan {
  Family family = Family::Ew;
  std::string func;
  std::vector<int64_t> grid;
  std::vector<Type> arg_types;   // memref args in signature order
  std::vector<std::string> arg_names;
  std::vector<std::string> notes;  // diagnostics (e.g. shared-contract notes)
  EwPlan ew;
  RowPlan rows;
  GemmPlan gemm;
  ConvPlan conv;
  TilePlan tile;
};

// Classifies ``f`` (throws Error(kUnsupported) with the reason otherwise).
Plan make_plan(const Module& m, const Func& f);

// Text of the plan for the stage dumps (stage 1..7 == the reference's
// xt_serialize .. nova_to_x1 slots).
std::string describe_plan(const Plan& p, int stage);

const char* family_name(Family f);

}  // namespace xt
