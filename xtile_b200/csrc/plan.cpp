// Classification of xt Block programs into B200 kernel families.
//
// Semantics restated from the reference:
//  * tile coordinate -> element start = index * tile dim (lib/xt/XTToNova.cpp:82-101);
//  * the grid enumerates every (x, y, z) Block (lib/xt/XTSerialize.cpp:68-84);
//  * matmul epilogue C = (A.B) * scale + bias [-> int8] is what
//    lib/nova/NovaOptimize.cpp:126-296 folds t*s+b and ftoi into;
//  * load_conv2d: zero-padded convolution of the halo slice
//    (lib/xt/XTToNova.cpp:103-142,353-437).
#include <algorithm>
#include <functional>
#include <map>
#include <set>
#include <sstream>

#include "plan.h"

namespace xt {

const char* family_name(Family f) {
  switch (f) {
    case Family::Ew: return "ew";
    case Family::Rows: return "rows";
    case Family::Gemm: return "gemm";
    case Family::Conv: return "conv";
    case Family::Tile: return "tile";
  }
  return "?";
}

namespace {

struct Coord {
  bool bid = false;
  int dim = -1;
  int64_t value = 0;
  bool operator==(const Coord& o) const { return bid == o.bid && dim == o.dim && value == o.value; }
};

// Linear-scan register file: a value owns its register from its definition
// to its last use; freeing is by owner, so a register handed to a later value
// is never released on behalf of an earlier one.
class RegFile {
 public:
  RegFile(int size, std::map<int, int> last_use) : owner_(size, -1), last_use_(std::move(last_use)) {}
  int alloc(int vid) {
    for (size_t r = 0; r < owner_.size(); ++r)
      if (owner_[r] < 0) {
        owner_[r] = vid;
        high_ = std::max(high_, static_cast<int>(r) + 1);
        return static_cast<int>(r);
      }
    return -1;
  }
  int get(int vid) const {
    for (size_t r = 0; r < owner_.size(); ++r)
      if (owner_[r] == vid) return static_cast<int>(r);
    throw Error(kUnsupported, "internal: value has no register");
  }
  bool has(int vid) const { return std::find(owner_.begin(), owner_.end(), vid) != owner_.end(); }
  // frees the registers of values whose last use is at or before op ``upto``
  void release_dead(int upto) {
    for (int& o : owner_)
      if (o >= 0) {
        auto it = last_use_.find(o);
        if (it == last_use_.end() || it->second <= upto) o = -1;
      }
  }
  int high_water() const { return high_; }

 private:
  std::vector<int> owner_;
  std::map<int, int> last_use_;
  int high_ = 0;
};

struct Access {
  int op = -1;                 // op index
  int arg = -1;                // memref argument position
  Type array;
  std::vector<int64_t> tile;
  std::vector<Coord> idx;
  int shared = 0;
};

class Classifier {
 public:
  Classifier(const Module& m, const Func& f) : m_(m), f_(f) {
    grid_ = func_grid(f);
    for (size_t k = 0; k < f.args.size(); ++k) arg_pos_[f.args[k]] = static_cast<int>(k);
  }

  Plan run() {
    if (f_.num_blocks != 1) unsupported("the function must have a single block");
    if (!f_.result_types.empty()) unsupported("the function must not return values");
    for (int a : f_.args)
      if (m_.value(a).type.kind != Type::MemRef) unsupported("every function argument must be a memref");
    Plan p;
    p.func = f_.name;
    p.grid = grid_;
    for (int a : f_.args) {
      p.arg_types.push_back(m_.value(a).type);
      p.arg_names.push_back(m_.value(a).name);
    }
    bool has_mm = false, has_conv = false;
    for (const Op& op : f_.ops) {
      has_mm |= op.name == "xt.matmul" || op.name == "xt.mma";
      has_conv |= op.name == "xt.load_conv2d";
    }
    collect_accesses();
    if (has_mm) {
      p.family = Family::Gemm;
      p.gemm = plan_gemm(p.notes);
    } else if (has_conv) {
      p.family = Family::Conv;
      p.conv = plan_conv();
    } else {
      std::string ew_why, rows_why;
      try {
        p.ew = plan_ew();
        p.family = Family::Ew;
        return p;
      } catch (const Error& e) {
        ew_why = e.what();
      }
      try {
        p.rows = plan_rows();
        p.family = Family::Rows;
        return p;
      } catch (const Error& e) {
        rows_why = e.what();
      }
      std::string tile_why;
      try {
        p.tile = plan_tile();
        p.family = Family::Tile;
        return p;
      } catch (const Error& e) {
        tile_why = e.what();
      }
      throw Error(kUnsupported, "no B200 kernel family matches @" + f_.name + ": as an elementwise map: " +
                                    ew_why + "; as a row program: " + rows_why + "; as a tile program: " + tile_why);
    }
    return p;
  }

 private:
  const Module& m_;
  const Func& f_;
  std::vector<int64_t> grid_;
  std::map<int, int> arg_pos_;
  std::map<int, Access> loads_;     // result value id -> access
  std::vector<Access> stores_;
  std::map<int, int> uses_;         // value id -> use count

  [[noreturn]] void unsupported(const std::string& why) const { throw Error(kUnsupported, why); }

  // value id -> index of the last op that reads it
  std::map<int, int> last_uses() const {
    std::map<int, int> last;
    for (size_t i = 0; i < f_.ops.size(); ++i)
      for (int v : f_.ops[i].operands) last[v] = static_cast<int>(i);
    return last;
  }

  const Op* def(int vid) const {
    int d = m_.value(vid).def_op;
    return d < 0 ? nullptr : &f_.ops[d];
  }

  Coord coord(int vid) const {
    const Op* op = def(vid);
    if (op && op->name == "xt.get_tile_block_id") {
      for (int k = 0; k < 3; ++k)
        if (op->results[k] == vid) return Coord{true, k, 0};
    }
    if (op && op->name == "arith.constant" && !op->is_dense && op->result_types[0].kind == Type::Scalar)
      return Coord{false, -1, op->ivalue};
    unsupported("tile coordinates must be xt.get_tile_block_id results or integer constants");
  }

  void collect_accesses() {
    for (size_t i = 0; i < f_.ops.size(); ++i) {
      const Op& op = f_.ops[i];
      for (int v : op.operands) uses_[v]++;
      if (op.name == "xt.load" || op.name == "xt.store") {
        Access a;
        a.op = static_cast<int>(i);
        bool is_store = op.name == "xt.store";
        int mem = op.operands[is_store ? 1 : 0];
        auto it = arg_pos_.find(mem);
        if (it == arg_pos_.end()) unsupported("loads and stores must address function arguments");
        a.arg = it->second;
        a.array = m_.value(mem).type;
        a.tile = is_store ? op.operand_types[0].shape : op.result_types[0].shape;
        for (size_t k = is_store ? 2 : 1; k < op.operands.size(); ++k) a.idx.push_back(coord(op.operands[k]));
        if (const Attr* s = find_attr(op.attrs, "shared")) a.shared = static_cast<int>(s->i);
        if (is_store) stores_.push_back(a);
        else loads_[op.results[0]] = a;
      }
    }
    if (stores_.empty()) unsupported("the program stores nothing");
  }

  // Elements [lo, hi) of one dim that the grid covers through coordinate c.
  std::pair<int64_t, int64_t> covered(const Coord& c, int64_t tile, int64_t dim) const {
    if (c.bid) return {0, std::min(grid_[c.dim] * tile, dim)};
    return {std::min(c.value * tile, dim), std::min((c.value + 1) * tile, dim)};
  }

  // ------------------------------------------------------------------ tile
  // Any Block program of loads, stores, elementwise ops with broadcasting,
  // reductions, reshape / transpose / permute and tensor constants.  Values
  // live in shared memory as f32 (int8 values are exact there and wrap on
  // add/sub/mul like the reference's int8 arithmetic).
  TilePlan plan_tile() {
    TilePlan p;
    std::map<int, int> val_of;  // SSA value id -> tile value index
    auto padded = [&](const std::vector<int64_t>& shape, int32_t (&out)[kTileRank]) {
      if (shape.size() > static_cast<size_t>(kTileRank)) unsupported("tile programs use rank <= 4 tiles");
      const int lead = kTileRank - static_cast<int>(shape.size());
      for (int d = 0; d < kTileRank; ++d) {
        const int64_t v = d < lead ? 1 : shape[d - lead];
        if (v <= 0 || v > (int64_t{1} << 30)) unsupported("tile and array dims must be in [1, 2^30]");
        out[d] = static_cast<int32_t>(v);
      }
      return lead;
    };
    // Shared-memory slots: a value's slot is freed after its last reader and
    // may then hold a later value that fits; an elementwise op may write its
    // result into the slot of a same-shaped operand it reads for the last
    // time (each element is read and written by the same thread at the same
    // index).  A permute folded into a store gets no slot: nothing writes it.
    struct Slot {
      int32_t offset;
      int64_t floats;
    };
    std::vector<Slot> free_slots;
    std::map<int, Slot> val_slot;  // tile value index -> its slot
    auto new_val = [&](int vid, const Type& t, int inplace = -1, bool no_slot = false) -> uint8_t {
      if (p.vals.size() == static_cast<size_t>(kTileMaxVals)) unsupported("the program has more than 16 tiles");
      if (t.elem != Elem::F32 && t.elem != Elem::I8 && t.elem != Elem::BF16) unsupported("unsupported element type");
      TileVal v{};
      padded(t.shape, v.shape);
      // rows padded to an odd length, so column walks (transpose, axis-0
      // reductions) touch distinct shared-memory banks
      const int64_t inner = v.shape[3] % 2 == 0 ? v.shape[3] + 1 : v.shape[3];
      const int64_t s2 = inner, s1 = s2 * v.shape[2], s0 = s1 * v.shape[1];
      const int64_t floats = s0 * v.shape[0];
      int64_t offset = -1;
      if (no_slot) {
        offset = 0;
      } else if (inplace >= 0) {
        const Slot sl = val_slot.at(inplace);
        val_slot.erase(inplace);  // the operand's slot passes to this value
        offset = sl.offset;
        val_slot[static_cast<int>(p.vals.size())] = sl;
      } else {
        int best = -1;
        for (size_t k = 0; k < free_slots.size(); ++k)
          if (free_slots[k].floats >= floats && (best < 0 || free_slots[k].floats < free_slots[best].floats))
            best = static_cast<int>(k);
        if (best >= 0) {
          offset = free_slots[best].offset;
          val_slot[static_cast<int>(p.vals.size())] = free_slots[best];
          free_slots.erase(free_slots.begin() + best);
        } else {
          offset = (static_cast<int64_t>(p.smem_floats) + 3) & ~int64_t{3};
          if (offset + floats > kTileSmemFloats) unsupported("the program's tiles exceed 192 KiB of shared memory");
          p.smem_floats = static_cast<int32_t>(offset + floats);
          val_slot[static_cast<int>(p.vals.size())] = Slot{static_cast<int32_t>(offset), floats};
        }
      }
      v.stride[3] = 1;
      v.stride[2] = static_cast<int32_t>(s2);
      v.stride[1] = static_cast<int32_t>(s1);
      v.stride[0] = static_cast<int32_t>(s0);
      v.numel = v.shape[0] * v.shape[1] * v.shape[2] * v.shape[3];
      v.offset = static_cast<int32_t>(offset);
      v.i8 = t.elem == Elem::I8;
      val_of[vid] = static_cast<int>(p.vals.size());
      p.vals.push_back(v);
      return static_cast<uint8_t>(p.vals.size() - 1);
    };
    auto val = [&](int vid) -> uint8_t {
      auto it = val_of.find(vid);
      if (it == val_of.end()) unsupported("a tile operand is not a tile value of the program");
      return static_cast<uint8_t>(it->second);
    };
    auto slot_of = [&](const Access& a) -> uint8_t {
      for (int i = 0; i < p.n_args; ++i)
        if (p.arg[i] == a.arg) return static_cast<uint8_t>(i);
      if (p.n_args == kTileMaxArgs) unsupported("the program addresses more than 8 arrays");
      if (a.array.elem != Elem::F32 && a.array.elem != Elem::I8 && a.array.elem != Elem::BF16)
        unsupported("unsupported array element type");
      const int i = p.n_args++;
      p.arg[i] = a.arg;
      p.arg_elem[i] = a.array.elem;
      padded(a.array.shape, p.arg_shape[i]);
      return static_cast<uint8_t>(i);
    };
    auto set_coords = [&](TileOp& t, const Access& a) {
      if (a.idx.size() != a.array.shape.size() || a.tile.size() != a.array.shape.size())
        unsupported("a tile's rank must match its array's rank");
      const int lead = kTileRank - static_cast<int>(a.idx.size());
      for (int d = 0; d < kTileRank; ++d) {
        t.coord_bid[d] = -1;
        t.coord[d] = 0;
        if (d < lead) continue;
        const Coord& c = a.idx[d - lead];
        if (c.bid) {
          t.coord_bid[d] = static_cast<int8_t>(c.dim);
        } else {
          if (c.value < 0 || c.value > (int64_t{1} << 30)) unsupported("tile coordinates must be in [0, 2^30]");
          t.coord[d] = static_cast<int32_t>(c.value);
        }
      }
    };
    std::map<int, const Access*> store_at;
    for (const Access& a : stores_) store_at[a.op] = &a;
    // Last reader of every value (op index).  A permute whose result only
    // feeds one store is folded into that store below, so its operand is
    // read at the store.
    std::map<int, int> last_use, n_uses, user;
    for (size_t i = 0; i < f_.ops.size(); ++i)
      for (int o : f_.ops[i].operands) {
        last_use[o] = static_cast<int>(i);
        ++n_uses[o];
        user[o] = static_cast<int>(i);
      }
    std::set<size_t> folded;  // permutes that become part of their store
    struct Fold {
      uint8_t src;
      uint8_t perm[kTileRank];
    };
    std::map<int, Fold> fold_of;  // folded permute's value index -> its operand and permutation
    for (size_t i = 0; i < f_.ops.size(); ++i) {
      const Op& op = f_.ops[i];
      if ((op.name != "xt.transpose" && op.name != "xt.permute") || op.results.empty()) continue;
      const int r = op.results[0];
      if (n_uses[r] == 1 && f_.ops[user[r]].name == "xt.store" && f_.ops[user[r]].operands[0] == r) {
        folded.insert(i);
        last_use[op.operands[0]] = std::max(last_use[op.operands[0]], user[r]);
      }
    }
    // frees the slots of the tile values whose last reader is op i
    auto release = [&](int i) {
      for (auto& kv : val_of) {
        auto it = last_use.find(kv.first);
        const int last = it == last_use.end() ? -1 : it->second;
        if (last <= i && val_slot.count(kv.second)) {
          free_slots.push_back(val_slot.at(kv.second));
          val_slot.erase(kv.second);
        }
      }
    };
    // an operand of op i whose slot the elementwise result may take over
    auto inplace_of = [&](const Op& op, int i, std::initializer_list<int> operand_idx) -> int {
      for (int k : operand_idx) {
        const int o = op.operands[k];
        auto it = val_of.find(o);
        if (it == val_of.end() || last_use[o] != i || !val_slot.count(it->second)) continue;
        if (op.operand_types[k].shape != op.result_types[0].shape) continue;
        return it->second;
      }
      return -1;
    };
    static const std::map<std::string, uint8_t> kUn = {
        {"xt.exp", kExp}, {"xt.cos", kCos}, {"xt.sin", kSin}, {"xt.reciprocal", kRecip}, {"xt.rsqrt", kRsqrt},
        {"xt.sigmoid", kSigmoid}, {"xt.tanh", kTanh}, {"xt.silu", kSilu}};
    static const std::map<std::string, uint8_t> kBin = {{"xt.add", kAdd}, {"xt.sub", kSub}, {"xt.mul", kMul}};
    for (size_t i = 0; i < f_.ops.size(); ++i) {
      const Op& op = f_.ops[i];
      const std::string& n = op.name;
      if (n == "xt.get_tile_block_id" || n == "func.return" || n == "return") continue;
      TileOp t{};
      if (n == "arith.constant") {
        if (op.result_types[0].kind != Type::Tensor) continue;  // a scalar tile coordinate
        if (!op.is_dense) unsupported("tensor constants must be dense splats");
        t.kind = kTConst;
        t.value = static_cast<float>(op.fvalue);
        t.dst = new_val(op.results[0], op.result_types[0]);
      } else if (n == "xt.load") {
        const Access& a = loads_.at(op.results[0]);
        t.kind = kTLoad;
        t.arg = slot_of(a);
        set_coords(t, a);
        t.dst = new_val(op.results[0], op.result_types[0]);
      } else if (n == "xt.store") {
        const Access& a = *store_at.at(static_cast<int>(i));
        t.kind = kTStore;
        t.a = val(op.operands[0]);
        auto fo = fold_of.find(t.a);
        if (fo != fold_of.end()) {
          // the stored tile is a folded permute: read its operand through the permuted strides
          t.code = 1;
          t.b = fo->second.src;
          for (int d = 0; d < kTileRank; ++d) t.perm[d] = fo->second.perm[d];
        }
        t.arg = slot_of(a);
        set_coords(t, a);
      } else if (kUn.count(n) || n == "xt.itof" || n == "xt.ftoi") {
        if (op.operand_types[0].shape != op.result_types[0].shape) unsupported("'" + n + "' changes the tile shape");
        if (n == "xt.itof" && op.operand_types[0].elem != Elem::I8) unsupported("itof expects i8");
        if (n == "xt.ftoi" && op.result_types[0].elem != Elem::I8) unsupported("ftoi produces i8");
        if (kUn.count(n) && op.operand_types[0].elem != Elem::F32) unsupported("'" + n + "' expects an f32 tile");
        t.kind = kTUnary;
        t.code = n == "xt.itof" ? static_cast<uint8_t>(kItof) : n == "xt.ftoi" ? static_cast<uint8_t>(kFtoi) : kUn.at(n);
        t.a = val(op.operands[0]);
        t.dst = new_val(op.results[0], op.result_types[0], inplace_of(op, static_cast<int>(i), {0}));
      } else if (kBin.count(n)) {
        t.kind = kTBinary;
        t.code = kBin.at(n);
        t.a = val(op.operands[0]);
        t.b = val(op.operands[1]);
        t.dst = new_val(op.results[0], op.result_types[0], inplace_of(op, static_cast<int>(i), {0, 1}));
        const TileVal &va = p.vals[t.a], &vb = p.vals[t.b], &vd = p.vals[t.dst];
        for (int d = 0; d < kTileRank; ++d)
          if ((va.shape[d] != vd.shape[d] && va.shape[d] != 1) || (vb.shape[d] != vd.shape[d] && vb.shape[d] != 1))
            unsupported("'" + n + "' operands do not broadcast to its result");
      } else if (n == "xt.reduce_max" || n == "xt.reduce_sum") {
        if (op.operand_types[0].elem != Elem::F32) unsupported("reductions are supported on f32 tiles");
        const Attr* ax = find_attr(op.attrs, "axis");
        const int rank = static_cast<int>(op.operand_types[0].shape.size());
        const int64_t axis = ax ? ax->i : rank - 1;
        if (axis < 0 || axis >= rank) unsupported("reduction axis out of range");
        t.kind = kTReduce;
        t.code = n == "xt.reduce_sum" ? 1 : 0;
        t.axis = static_cast<uint8_t>(kTileRank - rank + axis);
        t.a = val(op.operands[0]);
        t.dst = new_val(op.results[0], op.result_types[0]);
        for (int d = 0; d < kTileRank; ++d)
          if (p.vals[t.dst].shape[d] != (d == t.axis ? 1 : p.vals[t.a].shape[d]))
            unsupported("a reduction keeps every dim but the reduced one, which becomes 1");
      } else if (n == "xt.reshape") {
        t.kind = kTReshape;
        t.a = val(op.operands[0]);
        t.dst = new_val(op.results[0], op.result_types[0]);
        if (p.vals[t.a].numel != p.vals[t.dst].numel) unsupported("reshape must keep the element count");
      } else if (n == "xt.transpose" || n == "xt.permute") {
        const int rank = static_cast<int>(op.operand_types[0].shape.size());
        std::vector<int64_t> perm;
        if (n == "xt.transpose") {
          if (rank != 3) unsupported("transpose takes rank-3 tiles");
          perm = {0, 2, 1};
        } else {
          const Attr* pa = find_attr(op.attrs, "permutation");
          if (!pa) unsupported("permute needs a permutation");
          perm = pa->arr;
        }
        if (static_cast<int>(perm.size()) != rank) unsupported("the permutation must list every dim");
        std::vector<int64_t> sorted = perm;
        std::sort(sorted.begin(), sorted.end());
        for (int d = 0; d < rank; ++d)
          if (sorted[d] != d) unsupported("the permutation must use every dim once");
        t.kind = kTPermute;
        const int lead = kTileRank - rank;
        for (int d = 0; d < kTileRank; ++d)
          t.perm[d] = static_cast<uint8_t>(d < lead ? d : lead + perm[d - lead]);
        t.a = val(op.operands[0]);
        const bool fold = folded.count(i) > 0;
        t.dst = new_val(op.results[0], op.result_types[0], -1, fold);
        for (int d = 0; d < kTileRank; ++d)
          if (p.vals[t.dst].shape[d] != p.vals[t.a].shape[t.perm[d]])
            unsupported("the result shape must be the operand shape permuted");
        if (fold) {
          // no op: the one store of this value reads t.a through the permutation
          Fold f{t.a, {}};
          for (int d = 0; d < kTileRank; ++d) f.perm[d] = t.perm[d];
          fold_of[t.dst] = f;
          release(static_cast<int>(i));
          continue;
        }
      } else {
        unsupported("'" + n + "' is not supported in tile programs");
      }
      if (p.ops.size() == static_cast<size_t>(kTileMaxOps)) unsupported("the program has more than 32 tile ops");
      p.ops.push_back(t);
      release(static_cast<int>(i));
    }
    // (A permute whose result feeds nothing but one store was folded into
    // that store above: the store reads the permute's operand through the
    // permuted strides, code 1, which saves the kernel a pass over shared
    // memory and a CTA barrier per Block.)
    // Every Block stores tiles of its own: Blocks differing along any grid
    // axis must store to different tiles, or the result would depend on the
    // order in which Blocks run.
    for (const Access& a : stores_) {
      std::set<int> used;
      for (const Coord& c : a.idx)
        if (c.bid) {
          if (used.count(c.dim)) unsupported("a block axis may index only one dim of a stored tile");
          used.insert(c.dim);
        }
      for (int k = 0; k < static_cast<int>(grid_.size()); ++k)
        if (grid_[k] > 1 && !used.count(k))
          unsupported("Blocks along grid axis " + std::to_string(k) + " would store the same tile");
    }
    return p;
  }

  // ------------------------------------------------------------------ ew
  EwPlan plan_ew() {
    EwPlan p;
    const Access* ref = stores_.empty() ? nullptr : &stores_[0];
    auto same_map = [&](const Access& a) {
      if (a.tile != ref->tile || a.idx != ref->idx || a.array.shape != ref->array.shape)
        unsupported("loads and stores must use the same tile shape, index and array shape");
    };
    // A load of a [1, C] row at (0, j) with tiles (1, tn), beside [R, C]
    // arrays in (tm, tn) tiles at (i, j), broadcasts the row over the rows:
    // element (r, c) of the flat map reads element c of the row.
    auto row_bcast = [&](const Access& a) {
      return ref && ref->array.shape.size() == 2 && a.array.shape.size() == 2 && a.array.shape[0] == 1 &&
             a.array.shape[1] == ref->array.shape[1] && ref->array.shape[0] > 1 && a.tile.size() == 2 &&
             a.tile[0] == 1 && a.tile[1] == ref->tile[1] && !a.idx[0].bid && a.idx[0].value == 0 &&
             a.idx[1] == ref->idx[1];
    };
    if (!ref) unsupported("the program stores nothing");
    std::set<int> bcast_vals;  // SSA values loaded as row broadcasts, and values computed only from them
    for (auto& kv : loads_) {
      if (row_bcast(kv.second)) {
        bcast_vals.insert(kv.first);
        continue;
      }
      same_map(kv.second);
    }
    for (auto& s : stores_) same_map(s);
    // the grid must cover every element exactly once
    std::set<int> axes;
    for (size_t d = 0; d < ref->idx.size(); ++d) {
      const Coord& c = ref->idx[d];
      auto r = covered(c, ref->tile[d], ref->array.shape[d]);
      if (r.first != 0 || r.second != ref->array.shape[d])
        unsupported("the grid's tiles must cover the whole array");
      if (c.bid) {
        if (axes.count(c.dim)) unsupported("a block axis may index only one tile dimension");
        axes.insert(c.dim);
      }
    }
    p.shape = ref->array.shape;
    p.numel = ref->array.numel();
    if (!ref->idx.empty() && ref->idx[0].bid && ref->idx[0].dim == 0)
      p.bid0_span = ref->tile[0] * (p.numel / ref->array.shape[0]);

    RegFile regs(8, last_uses());
    auto alloc = [&](int vid) {
      int r = regs.alloc(vid);
      if (r < 0) unsupported("the program needs more than 8 live tiles");
      p.n_regs = std::max(p.n_regs, regs.high_water());
      return r;
    };
    std::map<int, int> in_slot;
    for (size_t i = 0; i < f_.ops.size(); ++i) {
      const Op& op = f_.ops[i];
      const std::string& n = op.name;
      if (n == "xt.get_tile_block_id" || n == "arith.constant" || n == "func.return" || n == "return") {
        if (n == "arith.constant" && op.is_dense) unsupported("tensor constants are not supported");
        continue;
      }
      auto reg = [&](int v) { return static_cast<uint8_t>(regs.get(v)); };
      regs.release_dead(static_cast<int>(i) - 1);
      if (n == "xt.load") {
        const Access& a = loads_.at(op.results[0]);
        Elem e = a.array.elem;
        if (e != Elem::F32 && e != Elem::I8 && e != Elem::BF16) unsupported("unsupported element type");
        const bool bc = bcast_vals.count(op.results[0]) > 0;
        auto it = in_slot.find(a.arg);
        int slot;
        if (it == in_slot.end()) {
          if (p.n_in == kMaxSlots) unsupported("too many input arrays");
          slot = p.n_in++;
          p.in_arg[slot] = a.arg;
          p.in_elem[slot] = e;
          p.in_bcast[slot] = bc;
          in_slot[a.arg] = slot;
        } else {
          slot = it->second;
          if (p.in_bcast[slot] != bc) unsupported("an array is loaded both as a row broadcast and as tiles");
        }
        if (bc) p.bcast_period = ref->array.shape[1];
        int r = alloc(op.results[0]);
        p.code.push_back({kLoad, static_cast<uint8_t>(r), static_cast<uint8_t>(slot), 0});
      } else if (n == "xt.store") {
        if (bcast_vals.count(op.operands[0])) unsupported("a row-broadcast value is stored");
        const Access* a = nullptr;
        for (auto& s : stores_) if (s.op == static_cast<int>(i)) a = &s;
        Elem e = a->array.elem;
        if (e != Elem::F32 && e != Elem::I8 && e != Elem::BF16) unsupported("unsupported element type");
        if (p.n_out == kMaxSlots) unsupported("too many stores");
        int slot = p.n_out++;
        p.out_arg[slot] = a->arg;
        p.out_elem[slot] = e;
        p.code.push_back({kStore, static_cast<uint8_t>(slot), reg(op.operands[0]), 0});
      } else {
        static const std::map<std::string, uint8_t> kOps = {
            {"xt.add", kAdd}, {"xt.sub", kSub}, {"xt.mul", kMul}, {"xt.exp", kExp},
            {"xt.cos", kCos}, {"xt.sin", kSin}, {"xt.reciprocal", kRecip}, {"xt.rsqrt", kRsqrt},
            {"xt.sigmoid", kSigmoid}, {"xt.tanh", kTanh}, {"xt.silu", kSilu},
            {"xt.itof", kItof}, {"xt.ftoi", kFtoi}};
        auto it = kOps.find(n);
        if (it == kOps.end()) unsupported("'" + n + "' is not an elementwise op");
        // an operand of the row-broadcast shape (1, tn) must hold broadcast
        // values; a result of that shape is one too
        const std::vector<int64_t> row_shape = {1, ref->tile.size() == 2 ? ref->tile[1] : -1};
        bool all_bcast = true;
        for (size_t k = 0; k < op.operands.size(); ++k) {
          const Type& t = op.operand_types[k];
          const bool bc = bcast_vals.count(op.operands[k]) > 0;
          all_bcast = all_bcast && bc;
          if (t.shape == op.result_types[0].shape && (!bc || t.shape == row_shape)) continue;
          if (bc && t.shape == row_shape && op.result_types[0].shape.size() == 2 &&
              op.result_types[0].shape[1] == row_shape[1])
            continue;
          unsupported("broadcasting ops are not elementwise");
        }
        if (all_bcast) {
          if (op.result_types[0].shape != row_shape) unsupported("broadcasting ops are not elementwise");
          bcast_vals.insert(op.results[0]);
        } else if (op.result_types[0].shape == row_shape && ref->tile[0] != 1) {
          unsupported("broadcasting ops are not elementwise");
        }
        bool binary = op.operands.size() == 2;
        if (binary && op.result_types[0].elem != Elem::F32)
          unsupported("elementwise arithmetic is supported on f32 tiles");
        if (n == "xt.itof" && op.operand_types[0].elem != Elem::I8) unsupported("itof expects i8");
        if (n == "xt.ftoi" && op.result_types[0].elem != Elem::I8) unsupported("ftoi produces i8");
        uint8_t a = reg(op.operands[0]);
        uint8_t b = binary ? reg(op.operands[1]) : 0;
        // operands dying at this op may give their register to its result
        regs.release_dead(static_cast<int>(i));
        int r = alloc(op.results[0]);
        p.code.push_back({it->second, static_cast<uint8_t>(r), a, b});
      }
      if (p.code.size() > static_cast<size_t>(kMaxInstr)) unsupported("the program is too long");
    }
    if (p.n_in == 0) unsupported("the program loads nothing");
    return p;
  }

  // ---------------------------------------------------------------- rows
  RowPlan plan_rows() {
    RowPlan p;
    int64_t R = -1, C = -1, tr = -1;
    int axis = -1;
    auto check = [&](const Access& a, bool* scalar) {
      if (a.array.rank() != 2) unsupported("row programs use rank-2 arrays");
      if (a.array.elem != Elem::F32) unsupported("row programs use f32 arrays");
      if (!a.idx[0].bid || a.idx[1].bid || a.idx[1].value != 0)
        unsupported("row tiles must be indexed (xt.bid(k), 0)");
      bool sc = a.array.shape[1] == 1;
      if (!sc && a.tile[1] != a.array.shape[1]) unsupported("row tiles must span whole rows");
      if (sc && a.tile[1] != 1) unsupported("per-row scalars must be (rows, 1) tiles");
      if (axis < 0) {
        axis = a.idx[0].dim;
        tr = a.tile[0];
        R = a.array.shape[0];
      }
      if (a.idx[0].dim != axis || a.tile[0] != tr || a.array.shape[0] != R)
        unsupported("all row tiles must share the row axis, tile height and row count");
      if (!sc) {
        if (C >= 0 && C != a.array.shape[1]) unsupported("all row arrays must have the same width");
        C = a.array.shape[1];
      }
      *scalar = sc;
    };
    for (auto& kv : loads_) { bool s; check(kv.second, &s); }
    for (auto& s : stores_) { bool sc; check(s, &sc); }
    if (C < 0) unsupported("the program has no full-row tile");
    p.rows = std::min(grid_[axis] * tr, R);
    p.cols = C;
    p.tile_rows = tr;
    p.row_axis = axis;

    // register allocation for row registers (v) and scalar registers (s)
    RegFile vregs(3, last_uses()), sregs(8, last_uses());
    auto is_row = [&](const Type& t) { return t.rank() == 2 && t.shape[1] == C && C != 1; };
    auto free_dead = [&](int i) {
      vregs.release_dead(i);
      sregs.release_dead(i);
    };
    auto alloc = [&](int vid, bool row) -> uint8_t {
      int r = (row ? vregs : sregs).alloc(vid);
      if (r < 0) unsupported(row ? "the row program needs more than 3 live rows" : "too many live row scalars");
      p.n_vregs = vregs.high_water();
      p.n_sregs = sregs.high_water();
      return static_cast<uint8_t>(r);
    };
    std::map<int, int> in_slot;
    for (size_t i = 0; i < f_.ops.size(); ++i) {
      const Op& op = f_.ops[i];
      const std::string& n = op.name;
      int ii = static_cast<int>(i);
      if (n == "xt.get_tile_block_id" || n == "func.return" || n == "return") continue;
      if (n == "arith.constant") {
        if (op.is_dense) unsupported("tensor constants are not supported");
        continue;
      }
      if (n == "xt.load") {
        const Access& a = loads_.at(op.results[0]);
        bool sc = a.array.shape[1] == 1;
        int slot;
        auto it = in_slot.find(a.arg);
        if (it == in_slot.end()) {
          if (p.n_in == kMaxSlots) unsupported("too many input arrays");
          slot = p.n_in++;
          p.in_arg[slot] = a.arg;
          p.in_is_scalar[slot] = sc;
          in_slot[a.arg] = slot;
        } else {
          slot = it->second;
        }
        free_dead(ii - 1);
        uint8_t r = alloc(op.results[0], !sc);
        p.code.push_back({sc ? kLoadScalar : kLoad, r, static_cast<uint8_t>(slot), 0});
        continue;
      }
      if (n == "xt.store") {
        const Access* a = nullptr;
        for (auto& s : stores_) if (s.op == ii) a = &s;
        bool sc = a->array.shape[1] == 1;
        if (p.n_out == kMaxSlots) unsupported("too many stores");
        int slot = p.n_out++;
        p.out_arg[slot] = a->arg;
        p.out_is_scalar[slot] = sc;
        uint8_t r = static_cast<uint8_t>(sc ? sregs.get(op.operands[0]) : vregs.get(op.operands[0]));
        p.code.push_back({sc ? kStoreScalar : kStore, static_cast<uint8_t>(slot), r, 0});
        continue;
      }
      const Type& res = op.result_types[0];
      if (res.elem != Elem::F32) unsupported("row programs compute in f32");
      auto operand_reg = [&](int v) -> uint8_t {
        return static_cast<uint8_t>(vregs.has(v) ? vregs.get(v) : sregs.get(v));
      };
      if (n == "xt.reduce_max" || n == "xt.reduce_sum") {
        const Attr* ax = find_attr(op.attrs, "axis");
        int64_t axis_v = ax->i < 0 ? ax->i + 2 : ax->i;
        if (axis_v != 1) unsupported("row programs reduce along axis 1 only");
        if (!is_row(op.operand_types[0])) unsupported("reductions must read a full row");
        uint8_t a = operand_reg(op.operands[0]);
        free_dead(ii);
        uint8_t r = alloc(op.results[0], false);
        p.code.push_back({n == "xt.reduce_max" ? kRowMax : kRowSum, r, a, 0});
        continue;
      }
      static const std::map<std::string, uint8_t> kBin = {{"xt.add", kAdd}, {"xt.sub", kSub}, {"xt.mul", kMul}};
      static const std::map<std::string, uint8_t> kUn = {
          {"xt.exp", kExp}, {"xt.cos", kCos}, {"xt.sin", kSin}, {"xt.reciprocal", kRecip},
          {"xt.rsqrt", kRsqrt}, {"xt.sigmoid", kSigmoid}, {"xt.tanh", kTanh}, {"xt.silu", kSilu}};
      if (kBin.count(n)) {
        bool lrow = is_row(op.operand_types[0]), rrow = is_row(op.operand_types[1]);
        uint8_t a = operand_reg(op.operands[0]), b = operand_reg(op.operands[1]);
        uint8_t opc;
        if (lrow && rrow) opc = kBin.at(n);
        else if (lrow && !rrow) opc = n == "xt.add" ? kBcastAdd : n == "xt.sub" ? kBcastSub : kBcastMul;
        else if (!lrow && !rrow) opc = kBin.at(n) | 0x80;
        else unsupported("a per-row scalar may only be the right operand of a row op");
        free_dead(ii);
        uint8_t r = alloc(op.results[0], lrow);
        p.code.push_back({opc, r, a, b});
        continue;
      }
      if (kUn.count(n)) {
        bool row = is_row(op.operand_types[0]);
        uint8_t a = operand_reg(op.operands[0]);
        free_dead(ii);
        uint8_t r = alloc(op.results[0], row);
        p.code.push_back({static_cast<uint8_t>(kUn.at(n) | (row ? 0 : 0x80)), r, a, 0});
        continue;
      }
      unsupported("'" + n + "' is not supported in row programs");
    }
    if (p.code.size() > static_cast<size_t>(kMaxInstr)) unsupported("the program is too long");
    if (row_cta_threads(C, std::max(p.n_vregs, 1)) == 0)
      unsupported("the program's live rows of " + std::to_string(C) + " elements exceed a CTA's registers");
    p.softmax = is_softmax_chain(p);
    return p;
  }

  // The softmax chain as plan_rows emits it for kernels/softmax.py and the
  // reciprocal form of test/python/dsl_convert.py:30-37: Load v; RowMax s<-v;
  // BcastSub v'<-v,s; Exp v''<-v'; RowSum s'<-v''; Recip(scalar) s''<-s';
  // BcastMul v'''<-v'',s''; Store v'''.
  static bool is_softmax_chain(const RowPlan& p) {
    if (p.code.size() != 8 || p.n_in != 1 || p.n_out != 1 || p.in_is_scalar[0] || p.out_is_scalar[0])
      return false;
    const Instr* c = p.code.data();
    return c[0].op == kLoad && c[1].op == kRowMax && c[1].a == c[0].dst && c[2].op == kBcastSub &&
           c[2].a == c[0].dst && c[2].b == c[1].dst && c[3].op == kExp && c[3].a == c[2].dst &&
           c[4].op == kRowSum && c[4].a == c[3].dst && c[5].op == (kRecip | 0x80) && c[5].a == c[4].dst &&
           c[6].op == kBcastMul && c[6].a == c[3].dst && c[6].b == c[5].dst && c[7].op == kStore &&
           c[7].a == c[6].dst;
  }

  // ---------------------------------------------------------------- gemm
  struct Term {
    const Access* a;
    const Access* b;
  };

  const Access& load_of(int vid, const char* what) {
    auto it = loads_.find(vid);
    if (it == loads_.end()) unsupported(std::string(what) + " must be loaded directly from an array");
    return it->second;
  }

  // Collects matmul terms of a sum tree (xt.add of matmuls) or an mma chain.
  void collect_terms(int vid, std::vector<Term>& terms, int* acc_vid) {
    const Op* op = def(vid);
    if (!op) unsupported("the matmul result must come from xt.matmul / xt.mma");
    if (uses_[vid] > 1) unsupported("intermediate matmul values may have only one use");
    if (op->name == "xt.matmul") {
      terms.push_back({&load_of(op->operands[0], "matmul lhs"), &load_of(op->operands[1], "matmul rhs")});
      return;
    }
    if (op->name == "xt.add" && op->operand_types[0] == op->operand_types[1]) {
      collect_terms(op->operands[0], terms, acc_vid);
      collect_terms(op->operands[1], terms, acc_vid);
      return;
    }
    if (op->name == "xt.mma") {
      terms.push_back({&load_of(op->operands[0], "mma lhs"), &load_of(op->operands[1], "mma rhs")});
      const Op* acc = def(op->operands[2]);
      if (acc && (acc->name == "xt.mma" || acc->name == "xt.matmul" || acc->name == "xt.add")) {
        collect_terms(op->operands[2], terms, acc_vid);
      } else {
        if (*acc_vid >= 0) unsupported("an mma chain may start from one accumulator tile");
        *acc_vid = op->operands[2];
      }
      return;
    }
    unsupported("'" + op->name + "' cannot feed the matmul accumulator");
  }

  GemmPlan plan_gemm(std::vector<std::string>& notes) {
    GemmPlan g;
    if (stores_.size() != 1) unsupported("a matmul program must store exactly one tile");
    const Access& st = stores_[0];
    const Op& store_op = f_.ops[st.op];
    int v = store_op.operands[0];
    if (st.array.rank() != 2) unsupported("matmul output must be rank 2");
    // walk back through the epilogue: [ftoi] <- (mul|add by row/scalar tile)*
    std::vector<EpiStep> rev;
    std::vector<const Access*> epi_loads;
    const Op* op = def(v);
    if (op && op->name == "xt.ftoi") {
      g.ftoi = true;
      v = op->operands[0];
      op = def(v);
    }
    while (op && (op->name == "xt.mul" || op->name == "xt.add")) {
      const Type& lt = op->operand_types[0];
      const Type& rt = op->operand_types[1];
      if (lt == rt) break;  // a tile + tile add: part of a K sum
      int other = op->operands[1];
      if (rt.shape != std::vector<int64_t>{1, rt.shape[1]} || (rt.shape[1] != lt.shape[1] && rt.shape[1] != 1))
        unsupported("epilogue operands must be (1, tn) rows or (1, 1) scalars");
      const Access& a = load_of(other, "epilogue operand");
      if (a.array.elem != Elem::F32) unsupported("epilogue rows must be f32");
      bool scalar = rt.shape[1] == 1;
      if (!scalar && a.array.shape[0] != 1) unsupported("epilogue rows must come from (1, N) arrays");
      EpiStep s;
      s.kind = op->name == "xt.mul" ? (scalar ? kEpiMulScalar : kEpiMulRow)
                                    : (scalar ? kEpiAddScalar : kEpiAddRow);
      s.arg = a.arg;
      rev.push_back(s);
      epi_loads.push_back(&a);
      if (uses_[v] > 1) unsupported("epilogue intermediates may have only one use");
      v = op->operands[0];
      op = def(v);
    }
    g.epi.assign(rev.rbegin(), rev.rend());
    std::vector<Term> terms;
    int acc_vid = -1;
    collect_terms(v, terms, &acc_vid);

    // all terms must share A/B arrays, M/N coordinates and tile shapes; their
    // K coordinates must enumerate 0..n-1
    const Access* a0 = terms[0].a;
    const Access* b0 = terms[0].b;
    std::set<int64_t> ks;
    for (const Term& t : terms) {
      if (t.a->arg != a0->arg || t.b->arg != b0->arg) unsupported("all matmul terms must read the same A and B");
      if (t.a->tile != a0->tile || t.b->tile != b0->tile) unsupported("all matmul terms must use the same tiles");
      if (!(t.a->idx[0] == a0->idx[0]) || !(t.b->idx[1] == b0->idx[1]))
        unsupported("all matmul terms must address the same output tile");
      if (t.a->idx[1].bid || t.b->idx[0].bid || t.a->idx[1].value != t.b->idx[0].value)
        unsupported("matmul K coordinates must be equal constants on A and B");
      ks.insert(t.a->idx[1].value);
    }
    if (static_cast<int64_t>(ks.size()) != static_cast<int64_t>(terms.size()) || *ks.begin() != 0 ||
        *ks.rbegin() != static_cast<int64_t>(terms.size()) - 1)
      unsupported("matmul K tiles must be 0 .. n-1, each once");
    const Type& A = a0->array;
    const Type& B = b0->array;
    if (A.elem != B.elem) unsupported("A and B must have the same element type");
    if (A.elem != Elem::BF16 && A.elem != Elem::I8)
      unsupported("tensor-core matmul needs bf16 or i8 operands (f32 has no exact tensor-core form)");
    g.ab_elem = A.elem;
    g.tm = a0->tile[0];
    g.tk = a0->tile[1];
    g.tn = b0->tile[1];
    g.k_steps = static_cast<int>(terms.size());
    g.a_arg = a0->arg;
    g.b_arg = b0->arg;
    g.c_arg = st.arg;
    g.c_elem = st.array.elem;
    if (g.ftoi != (g.c_elem == Elem::I8)) unsupported("an int8 result needs astype(int8) and vice versa");
    if (g.c_elem != Elem::F32 && g.c_elem != Elem::I8) unsupported("matmul output must be f32 or i8");
    const Coord& mi = a0->idx[0];
    const Coord& nj = b0->idx[1];
    if (!(st.idx[0] == mi) || !(st.idx[1] == nj)) unsupported("the store must use the A row and B column coordinates");
    if (st.tile[0] != g.tm || st.tile[1] != g.tn) unsupported("the stored tile must be tm x tn");
    if (mi.bid && nj.bid && mi.dim == nj.dim) unsupported("M and N tiles must use different block axes");
    if (!mi.bid && mi.value != 0) unsupported("a constant M coordinate must be 0");
    if (!nj.bid && nj.value != 0) unsupported("a constant N coordinate must be 0");
    g.m_axis = mi.bid ? mi.dim : -1;
    g.n_axis = nj.bid ? nj.dim : -1;
    g.M = std::min((mi.bid ? grid_[mi.dim] : 1) * g.tm, A.shape[0]);
    g.N = std::min((nj.bid ? grid_[nj.dim] : 1) * g.tn, B.shape[1]);
    g.K = std::min(g.k_steps * g.tk, std::min(A.shape[1], B.shape[0]));
    if (st.array.shape[0] < g.M || st.array.shape[1] < g.N) unsupported("output array too small");
    g.lda = A.shape[1];
    g.ldb = B.shape[1];
    g.ldc = st.array.shape[1];
    int align = A.elem == Elem::BF16 ? 8 : 16;  // 16-byte TMA strides
    if (g.lda % align || g.ldb % align)
      unsupported("A and B rows must be multiples of 16 bytes for TMA");
    if (acc_vid >= 0) {
      const Access& acc = load_of(acc_vid, "mma accumulator");
      if (acc.array.elem != Elem::F32 || acc.tile != st.tile || !(acc.idx == st.idx))
        unsupported("the mma accumulator must be the f32 output tile");
      g.acc_arg = acc.arg;
    }
    for (const Access* e : epi_loads) {
      bool scalar = e->tile[1] == 1 && g.tn != 1;
      if (e->idx[0].bid || e->idx[0].value != 0) unsupported("epilogue rows must be indexed (0, ...)");
      if (scalar) {
        if (e->idx[1].bid || e->idx[1].value != 0) unsupported("epilogue scalars must be indexed (0, 0)");
      } else if (!(e->idx[1] == nj) || e->tile[1] != g.tn || e->array.shape[1] < g.N) {
        unsupported("epilogue rows must be indexed by the B column coordinate");
      }
    }
    // shared=k is a promise that the tile is the same for blocks that agree
    // on axes >= k; note programs whose index breaks it (every load still
    // reads the tile its index names)
    for (auto& kv : loads_) {
      const Access& a = kv.second;
      if (a.shared > 0)
        for (const Coord& c : a.idx)
          if (c.bid && c.dim < a.shared)
            notes.push_back("shared=" + std::to_string(a.shared) + " load of %" +
                            m_.value(f_.args[a.arg]).name + " is indexed by xt.bid(" +
                            std::to_string(c.dim) + "): loaded per block by its index");
    }
    return g;
  }

  // ---------------------------------------------------------------- conv
  ConvPlan plan_conv() {
    ConvPlan c;
    if (stores_.size() != 1) unsupported("a conv program must store exactly one tile");
    const Access& st = stores_[0];
    const Op* op = def(f_.ops[st.op].operands[0]);
    if (!op || op->name != "xt.load_conv2d") unsupported("the stored tile must be the load_conv2d result");
    const Access& filt = load_of(op->operands[1], "the conv filter");
    auto src = arg_pos_.find(op->operands[0]);
    if (src == arg_pos_.end()) unsupported("the conv source must be a function argument");
    const Type& in = op->operand_types[0];
    const Type& ft = op->operand_types[1];
    const Type& res = op->result_types[0];
    for (const Coord& k : filt.idx)
      if (k.bid || k.value != 0) unsupported("the filter must be loaded whole at index 0");
    if (filt.tile != filt.array.shape) unsupported("the filter must be loaded whole");
    const Attr* g = find_attr(op->attrs, "group");
    if (g && g->i != 1) unsupported("grouped convolution is not supported");
    std::vector<Coord> idx;
    for (int k = 2; k < 6; ++k) idx.push_back(coord(op->operands[k]));
    if (idx[3].bid || idx[3].value != 0) unsupported("the channel coordinate must be 0");
    if (!(idx == st.idx)) unsupported("the store must use the load_conv2d coordinates");
    if (res.shape[3] != ft.shape[3]) unsupported("the result must hold every filter output channel");
    if (in.elem != Elem::BF16 && in.elem != Elem::I8)
      unsupported("the tensor-core conv takes bf16 or int8 input and filter");
    if (st.array.elem != Elem::F32) unsupported("the conv output must be f32");
    c.in_arg = src->second;
    c.filt_arg = filt.arg;
    c.out_arg = st.arg;
    c.elem = in.elem;
    c.N = in.shape[0];
    c.H = in.shape[1];
    c.W = in.shape[2];
    c.C = in.shape[3];
    c.KH = ft.shape[0];
    c.KW = ft.shape[1];
    c.KO = ft.shape[3];
    const Attr* pad = find_attr(op->attrs, "pad");
    const Attr* stride = find_attr(op->attrs, "stride");
    const Attr* dil = find_attr(op->attrs, "dilation");
    c.pad_t = pad->arr[0];
    c.pad_l = pad->arr[1];
    c.stride_h = stride->arr[0];
    c.stride_w = stride->arr[1];
    c.dil_h = dil->arr[0];
    c.dil_w = dil->arr[1];
    c.tb = res.shape[0];
    c.th = res.shape[1];
    c.tw = res.shape[2];
    const Type& out = st.array;
    c.out_h = out.shape[1];
    c.out_w = out.shape[2];
    c.out_c = out.shape[3];
    auto cov = [&](const Coord& k, int64_t tile, int64_t dim) {
      auto r = covered(k, tile, dim);
      if (r.first != 0) unsupported("conv tiles must start at the array origin");
      return r.second;
    };
    c.ON = cov(idx[0], c.tb, std::min(c.N, out.shape[0]));
    c.OH = cov(idx[1], c.th, out.shape[1]);
    c.OW = cov(idx[2], c.tw, out.shape[2]);
    c.OC = c.KO;
    c.n_axis = idx[0].bid ? idx[0].dim : -1;
    const int64_t eb = elem_bytes(c.elem);
    if ((c.C * eb) % 16) unsupported("input channel rows must be multiples of 16 bytes (TMA strides)");
    if (c.KO % 32 || c.KO > 256) unsupported("output channels must be a multiple of 32, at most 256");
    if (c.out_c % 4) unsupported("output channel rows must be multiples of 16 bytes (TMA stores)");
    if (c.stride_h != 1 || c.stride_w != 1) unsupported("strided convolution is not supported yet");
    return c;
  }
};

}  // namespace

Plan make_plan(const Module& m, const Func& f) {
  Classifier c(m, f);
  return c.run();
}

std::string describe_plan(const Plan& p, int stage) {
  std::ostringstream os;
  auto arr = [&](int arg) { return "%" + p.arg_names.at(arg); };
  os << "  // b200 @" << p.func << ": family " << family_name(p.family) << ", grid [" << p.grid[0] << ", "
     << p.grid[1] << ", " << p.grid[2] << "]\n";
  if (stage >= 1) {
    os << "  //   xt_serialize -> every (x, y, z) Block maps onto the CUDA grid; no unrolling\n";
  }
  if (stage >= 2) {
    switch (p.family) {
      case Family::Ew:
        os << "  //   xt_to_nova -> ew: " << p.ew.numel << " elements, " << p.ew.n_in << " inputs, "
           << p.ew.n_out << " outputs, " << p.ew.code.size() << " register ops\n";
        break;
      case Family::Rows:
        os << "  //   xt_to_nova -> rows: " << p.rows.rows << " rows x " << p.rows.cols << ", "
           << p.rows.code.size() << " row ops (reductions along axis 1)\n";
        break;
      case Family::Gemm:
        os << "  //   xt_to_nova -> gemm: M " << p.gemm.M << " N " << p.gemm.N << " K " << p.gemm.K << " ("
           << elem_name(p.gemm.ab_elem) << " -> " << elem_name(p.gemm.c_elem) << "), A " << arr(p.gemm.a_arg)
           << " B " << arr(p.gemm.b_arg) << " C " << arr(p.gemm.c_arg) << ", block tile " << p.gemm.tm << "x"
           << p.gemm.tn << "x" << p.gemm.tk << " x" << p.gemm.k_steps << "\n";
        break;
      case Family::Conv:
        os << "  //   xt_to_nova -> conv: implicit GEMM M " << p.conv.ON * p.conv.OH * p.conv.OW << " N "
           << p.conv.OC << " K " << p.conv.KH * p.conv.KW * p.conv.C << ", pad [" << p.conv.pad_t << ", "
           << p.conv.pad_l << "]\n";
        break;
      case Family::Tile:
        os << "  //   xt_to_nova -> tile: one CTA per Block, " << p.tile.vals.size() << " tiles in "
           << (p.tile.smem_floats * 4 + 1023) / 1024 << " KiB of shared memory, " << p.tile.ops.size()
           << " tile ops\n";
        break;
    }
  }
  if (stage >= 3 && p.family == Family::Gemm) {
    os << "  //   nova_optimize -> epilogue:";
    if (p.gemm.acc_arg >= 0) os << " + " << arr(p.gemm.acc_arg);
    for (const EpiStep& s : p.gemm.epi)
      os << (s.kind == kEpiMulRow || s.kind == kEpiMulScalar ? " * " : " + ") << arr(s.arg);
    if (p.gemm.ftoi) os << " -> i8 (round half even, saturate)";
    os << "\n";
  }
  if (stage >= 3 && (p.family == Family::Ew || p.family == Family::Rows)) {
    // the register program the ew / rows kernels are generated from
    static const char* kNames[] = {"?", "load", "store", "add", "sub", "mul", "exp", "cos", "sin",
                                   "recip", "rsqrt", "sigmoid", "tanh", "silu", "itof", "ftoi",
                                   "bcast_add", "bcast_sub", "bcast_mul", "rowmax", "rowsum",
                                   "load_scalar", "store_scalar"};
    const bool rows = p.family == Family::Rows;
    const std::vector<Instr>& code = rows ? p.rows.code : p.ew.code;
    const int* in_arg = rows ? p.rows.in_arg : p.ew.in_arg;
    const int* out_arg = rows ? p.rows.out_arg : p.ew.out_arg;
    auto reg = [&](uint8_t op, int r, bool operand_b) {
      if (!rows) return "r" + std::to_string(r);
      uint8_t o = op & 0x7f;
      bool scalar = (op & 0x80) || o == kRowMax || o == kRowSum || o == kLoadScalar ||
                    (operand_b && (o == kBcastAdd || o == kBcastSub || o == kBcastMul));
      return (scalar ? "s" : "v") + std::to_string(r);
    };
    os << "  //   nova_optimize -> register program (" << code.size() << " ops):\n";
    for (const Instr& ins : code) {
      uint8_t o = ins.op & 0x7f;
      os << "  //     ";
      if (o == kLoad || o == kLoadScalar) {
        os << (o == kLoadScalar ? "s" : (rows ? "v" : "r")) << int(ins.dst) << " = " << kNames[o] << " "
           << arr(in_arg[ins.a]) << "\n";
      } else if (o == kStore || o == kStoreScalar) {
        os << kNames[o] << " " << arr(out_arg[ins.dst]) << " <- "
           << (o == kStoreScalar ? "s" : (rows ? "v" : "r")) << int(ins.a) << "\n";
      } else if (o == kRowMax || o == kRowSum) {
        os << "s" << int(ins.dst) << " = " << kNames[o] << " v" << int(ins.a) << "\n";
      } else {
        bool binary = o == kAdd || o == kSub || o == kMul || o == kBcastAdd || o == kBcastSub || o == kBcastMul;
        bool scalar_dst = (ins.op & 0x80) != 0;
        os << (rows ? (scalar_dst ? "s" : "v") : "r") << int(ins.dst) << " = " << kNames[o] << " "
           << reg(ins.op, ins.a, false);
        if (binary) os << ", " << reg(ins.op, ins.b, true);
        os << "\n";
      }
    }
  }
  // rows: one warp per row up to 2048 columns while a lane holds the live
  // rows in 160 values (the generated kernels' rule), else one CTA per row
  const int n_v = std::max(p.rows.n_vregs, 1);
  const int row_cta = p.family == Family::Rows && !row_warp_fits(p.rows.cols, n_v)
                          ? row_cta_threads(p.rows.cols, n_v)
                          : 0;
  if (stage >= 4) {
    std::string threads;
    switch (p.family) {
      case Family::Gemm:
      case Family::Conv:
        threads = "warp 0 TMA producer, MMA issuer warp(s), TMEM epilogue warps";
        break;
      case Family::Rows:
        threads = row_cta ? "one CTA of " + std::to_string(row_cta) + " threads per row" : "one warp per row";
        break;
      case Family::Tile:
        threads = "one CTA per Block, loops of its threads over each op's tile";
        break;
      default:
        threads = "grid-stride, 8 elements per thread per step";
    }
    os << "  //   nova_threading -> " << threads << "\n";
  }
  if (stage >= 5) {
    const char* sync = p.family == Family::Gemm || p.family == Family::Conv
                           ? "mbarrier ring (full/empty per stage) + TMEM full/empty, bounded waits"
                       : p.family == Family::Tile ? "CTA barriers between ops that share shared memory"
                       : row_cta ? "CTA barriers in the row reductions"
                                 : "none (blocks are independent)";
    os << "  //   nova_barrier -> " << sync << "\n";
  }
  if (stage >= 6) {
    std::string mem;
    switch (p.family) {
      case Family::Gemm:
        mem = "4 smem stages of A 128x64 + B 64x256 (192 KiB), TMEM 512 columns";
        break;
      case Family::Conv:
        mem = "smem ring of shifted input tiles + resident filter, TMEM accumulator";
        break;
      case Family::Tile:
        mem = "tile slots in " + std::to_string((p.tile.smem_floats * 4 + 1023) / 1024) + " KiB of shared memory";
        break;
      default:
        mem = "registers only";
    }
    os << "  //   nova_allocate -> " << mem << "\n";
  }
  if (stage >= 7) os << "  //   nova_to_x1 -> launch via xt_launch (sm_100a)\n";
  for (const std::string& n : p.notes) os << "  //   note: " << n << "\n";
  return os.str();
}

}  // namespace xt
