//===- DsTransformPassB200.cpp - DS pass retargeted to libds_b200 -----------===//
//
// The reference's DsTransformPass (stablehlo_pass/DsTransformPass.cpp) turns
// float tensor arithmetic into double-single arithmetic inlined as StableHLO
// ops.  This pass applies the same lowering rules to the same operations but
// emits custom calls to libds_b200's targets, bound by adapters/ds_b200_ffi.cc:
//
//   add / subtract / multiply / negate (:282-321), with the constants and
//   broadcast_in_dim operands they read (:244-279)
//       -> one @ds_fused call per single-use tree of such operations, the tree
//          carried as data (one generated kernel per tree, bit-identical to the
//          per-operation DS lowering);
//   reduce with a one-operation add / subtract / multiply body (:376-448)
//       -> @ds_reduce_f64 {dimensions, body};
//   dot_general (:337-370), any dimension numbers
//       -> @ds_dot_general_f64 {lhs/rhs_batching_dimensions,
//          lhs/rhs_contracting_dimensions, algorithm}.
//
// Operations nested in while / if / case regions are rewritten in place
// (the reference's pass leaves nested regions for later); a tree never
// absorbs a producer of another block, so nothing moves into a loop body.
// The scalar bodies of reduce-like operations are left alone.
//
// Values between rewritten operations stay f64 (8 bytes, like the
// reference's hi/lo pair, and 53 bits instead of 48): an f32 operand is
// widened where it enters and a result narrowed back where an operation
// this pass leaves alone, or the return, reads it; a narrowing followed by
// a widening between two rewritten operations is folded away at the end,
// so the pair never loses bits in between (the reference's dsMap).  The
// function's signature is unchanged.  Custom calls use the typed FFI
// (api_version 4) with a dictionary backend_config.
//
// Built by adapters/CMakeLists.txt against an MLIR + StableHLO install
// (the reference's toolchain); this repository's image has neither.  The
// same rules run on torch programs in ds_b200/transform.py.
//
//===----------------------------------------------------------------------===//

#include <optional>

#include "llvm/ADT/DenseMap.h"
#include "llvm/ADT/DenseSet.h"
#include "llvm/ADT/STLExtras.h"
#include "llvm/ADT/SmallVector.h"
#include "mlir/Dialect/Func/IR/FuncOps.h"
#include "mlir/IR/Builders.h"
#include "mlir/IR/BuiltinAttributes.h"
#include "mlir/IR/BuiltinTypes.h"
#include "mlir/Pass/Pass.h"
#include "mlir/Pass/PassRegistry.h"
#include "stablehlo/dialect/StablehloOps.h"

using namespace mlir;

namespace {

// ds_fused_op codes and input / output kinds (include/ds_b200.h).
enum FusedCode : int32_t { kInput = 0, kConst = 1, kAdd = 2, kSub = 3, kMul = 4, kNeg = 5 };
enum FusedKind : int32_t { kKindF64 = 0, kKindF32 = 1 };
enum ReduceBody : int32_t { kBodyAdd = 0, kBodySub = 1, kBodyMul = 2 };
constexpr int kMaxOps = 256;     // ds_fused_run's limits
constexpr int kMaxInputs = 16;

constexpr llvm::StringLiteral kWiden = "ds_b200.widen";
constexpr llvm::StringLiteral kNarrow = "ds_b200.narrow";

bool isFloatTensor(Type t) {
  auto r = dyn_cast<RankedTensorType>(t);
  return r && (r.getElementType().isF32() || r.getElementType().isF64());
}

RankedTensorType withF64(Type t) {
  auto r = cast<RankedTensorType>(t);
  return RankedTensorType::get(r.getShape(), Float64Type::get(t.getContext()));
}

bool isElementwise(Operation* op) {
  return isa<stablehlo::AddOp, stablehlo::SubtractOp, stablehlo::MulOp, stablehlo::NegOp>(op) &&
         isFloatTensor(op->getResult(0).getType());
}

// A splat float constant's value.
std::optional<double> splatValue(Operation* op) {
  auto c = dyn_cast_or_null<stablehlo::ConstantOp>(op);
  if (!c || !isFloatTensor(c.getResult().getType())) return std::nullopt;
  auto v = dyn_cast<DenseElementsAttr>(c.getValue());
  if (!v || !v.isSplat()) return std::nullopt;
  return v.getSplatValue<APFloat>().convertToDouble();
}

// broadcast_in_dim that maps its operand onto the trailing dimensions of the
// result in order (numpy's broadcasting, which ds_fused applies itself).
Value numpyBroadcastSource(Operation* op) {
  auto bc = dyn_cast_or_null<stablehlo::BroadcastInDimOp>(op);
  if (!bc) return nullptr;
  auto in = cast<RankedTensorType>(bc.getOperand().getType());
  auto out = cast<RankedTensorType>(bc.getResult().getType());
  ArrayRef<int64_t> dims = bc.getBroadcastDimensions();
  const int64_t lead = out.getRank() - in.getRank();
  for (int64_t i = 0; i < in.getRank(); ++i) {
    if (dims[i] != lead + i) return nullptr;
    if (in.getDimSize(i) != 1 && in.getDimSize(i) != out.getDimSize(lead + i)) return nullptr;
  }
  return bc.getOperand();
}

// The body of a reduce the pass rewrites: acc = acc <op> x, one operation.
std::optional<int32_t> reduceBody(stablehlo::ReduceOp r) {
  Block& blk = r.getBody().front();
  if (blk.getNumArguments() != 2 || !llvm::hasSingleElement(blk.without_terminator()))
    return std::nullopt;
  Operation& op = blk.front();
  auto ret = dyn_cast<stablehlo::ReturnOp>(blk.getTerminator());
  if (!ret || ret->getNumOperands() != 1 || ret->getOperand(0) != op.getResult(0) ||
      op.getNumOperands() != 2)
    return std::nullopt;
  const bool inOrder = op.getOperand(0) == blk.getArgument(0) &&
                       op.getOperand(1) == blk.getArgument(1);
  const bool swapped = op.getOperand(0) == blk.getArgument(1) &&
                       op.getOperand(1) == blk.getArgument(0);
  if (isa<stablehlo::AddOp>(op) && (inOrder || swapped)) return kBodyAdd;
  if (isa<stablehlo::MulOp>(op) && (inOrder || swapped)) return kBodyMul;
  if (isa<stablehlo::SubtractOp>(op) && inOrder) return kBodySub;
  return std::nullopt;
}

// Operations in the function body, or nested only in control flow (while,
// if, case: the reference's "nested regions" next step) are rewritten.  The
// scalar computations of reduce-like operations (reduce, reduce_window,
// scatter, sort, ...) are not: only a reduce itself is.
bool inRewritableRegion(Operation* op) {
  for (Operation* p = op->getParentOp(); p && !isa<func::FuncOp>(p); p = p->getParentOp())
    if (!isa<stablehlo::WhileOp, stablehlo::IfOp, stablehlo::CaseOp>(p)) return false;
  return true;
}

bool isCandidate(Operation* op) {
  if (!op || !inRewritableRegion(op)) return false;
  if (isElementwise(op)) return true;
  if (auto d = dyn_cast<stablehlo::DotGeneralOp>(op))
    return isFloatTensor(d.getLhs().getType()) && isFloatTensor(d.getRhs().getType()) &&
           isFloatTensor(d.getResult().getType());
  if (auto r = dyn_cast<stablehlo::ReduceOp>(op))
    return r.getInputs().size() == 1 && isFloatTensor(r.getInputs()[0].getType()) &&
           reduceBody(r).has_value();
  return false;
}

// f64 view of an operand: f64 values as they are; f32 ones through a marked
// convert (exact).
Value widen(OpBuilder& b, Location loc, Value v) {
  auto t = cast<RankedTensorType>(v.getType());
  if (t.getElementType().isF64()) return v;
  auto c = b.create<stablehlo::ConvertOp>(loc, withF64(t), v);
  c->setAttr(kWiden, b.getUnitAttr());
  return c.getResult();
}

// The rewritten f64 result in the original element type.
Value narrow(OpBuilder& b, Location loc, Value v64, Type orig) {
  if (cast<RankedTensorType>(orig).getElementType().isF64()) return v64;
  auto c = b.create<stablehlo::ConvertOp>(loc, orig, v64);
  c->setAttr(kNarrow, b.getUnitAttr());
  return c.getResult();
}

Value customCall(OpBuilder& b, Location loc, StringRef target, Type result, ValueRange operands,
                 ArrayRef<NamedAttribute> config) {
  OperationState st(loc, stablehlo::CustomCallOp::getOperationName());
  st.addOperands(operands);
  st.addTypes(result);
  st.addAttribute("call_target_name", b.getStringAttr(target));
  st.addAttribute("api_version",
                  stablehlo::CustomCallApiVersionAttr::get(
                      b.getContext(), stablehlo::CustomCallApiVersion::API_VERSION_TYPED_FFI));
  st.addAttribute("backend_config", b.getDictionaryAttr(config));
  return b.create(st)->getResult(0);
}

// One elementwise tree as a ds_fused program.
struct Program {
  SmallVector<int32_t> codes, a, b;
  SmallVector<double> values;
  SmallVector<Value> inputs;
  SmallVector<int32_t> kinds;
  llvm::DenseMap<Value, int32_t> opOf;  // value -> index of its operation
  SmallVector<Operation*> absorbed;     // tree operations, operands first

  int32_t push(int32_t code, int32_t x, int32_t y, double v) {
    codes.push_back(code);
    a.push_back(x);
    b.push_back(y);
    values.push_back(v);
    return static_cast<int32_t>(codes.size()) - 1;
  }
};

class ProgramBuilder {
 public:
  ProgramBuilder(OpBuilder& b, Location loc, Block* block,
                 const llvm::DenseSet<Operation*>& done)
      : b_(b), loc_(loc), block_(block), done_(done) {}

  // Index of the operation producing v, absorbing single-use elementwise
  // producers of the root's own block when `absorb` (a producer outside a
  // loop body stays outside it); -1 when the program would exceed its
  // limits.
  int32_t build(Program& p, Value v, bool absorb) {
    if (auto it = p.opOf.find(v); it != p.opOf.end()) return it->second;
    if (static_cast<int>(p.codes.size()) + 1 > kMaxOps) return -1;
    Operation* def = v.getDefiningOp();
    int32_t id;
    if (auto c = splatValue(def)) {
      id = p.push(kConst, 0, 0, *c);
    } else if (absorb && def && def->getBlock() == block_ && isCandidate(def) && v.hasOneUse() &&
               !done_.contains(def) && isElementwise(def)) {
      const int32_t x = build(p, def->getOperand(0), absorb);
      if (x < 0) return -1;
      int32_t y = 0;
      if (def->getNumOperands() == 2 && (y = build(p, def->getOperand(1), absorb)) < 0) return -1;
      if (static_cast<int>(p.codes.size()) + 1 > kMaxOps) return -1;
      const int32_t code = isa<stablehlo::AddOp>(def)        ? kAdd
                           : isa<stablehlo::SubtractOp>(def) ? kSub
                           : isa<stablehlo::MulOp>(def)      ? kMul
                                                             : kNeg;
      id = p.push(code, x, y, 0.0);
      p.absorbed.push_back(def);
    } else {
      Value src = numpyBroadcastSource(def);
      if (!src || !isFloatTensor(src.getType())) src = v;
      if (static_cast<int>(p.inputs.size()) == kMaxInputs) return -1;
      // a value another rewrite will replace enters widened (the final fold
      // then hands over its f64 form); others enter as they are
      Value in = isCandidate(src.getDefiningOp()) ? widen(b_, loc_, src) : src;
      const bool f64 = cast<RankedTensorType>(in.getType()).getElementType().isF64();
      p.inputs.push_back(in);
      p.kinds.push_back(f64 ? kKindF64 : kKindF32);
      id = p.push(kInput, static_cast<int32_t>(p.inputs.size()) - 1, 0, 0.0);
    }
    p.opOf[v] = id;
    return id;
  }

 private:
  OpBuilder& b_;
  Location loc_;
  Block* block_;
  const llvm::DenseSet<Operation*>& done_;
};

struct DsTransformB200Pass
    : public PassWrapper<DsTransformB200Pass, OperationPass<func::FuncOp>> {
  MLIR_DEFINE_EXPLICIT_INTERNAL_INLINE_TYPE_ID(DsTransformB200Pass)

  StringRef getArgument() const final { return "ds-transform-b200"; }
  StringRef getDescription() const final {
    return "Lower float add/sub/mul/neg trees, reduce and dot_general to libds_b200 custom "
           "calls (double-single arithmetic on B200)";
  }

  void runOnOperation() final {
    func::FuncOp func = getOperation();
    SmallVector<Operation*> ops;
    func.walk([&](Operation* op) {
      if (isCandidate(op)) ops.push_back(op);
    });
    llvm::DenseSet<Operation*> done;
    // Consumers before producers: a tree's root is met before the
    // operations it absorbs.
    for (Operation* op : llvm::reverse(ops)) {
      if (done.contains(op)) continue;
      OpBuilder b(op);
      if (auto d = dyn_cast<stablehlo::DotGeneralOp>(op)) rewriteDot(b, d);
      else if (auto r = dyn_cast<stablehlo::ReduceOp>(op)) rewriteReduce(b, r);
      else rewriteTree(b, op, done);
      done.insert(op);
    }
    foldWidenedNarrowing(func);
  }

  void replace(OpBuilder& b, Operation* op, Value v64) {
    Value out = narrow(b, op->getLoc(), v64, op->getResult(0).getType());
    op->getResult(0).replaceAllUsesWith(out);
    op->erase();
  }

  void rewriteDot(OpBuilder& b, stablehlo::DotGeneralOp d) {
    Location loc = d.getLoc();
    auto dn = d.getDotDimensionNumbers();
    SmallVector<NamedAttribute> cfg = {
        b.getNamedAttr("lhs_batching_dimensions",
                       b.getDenseI64ArrayAttr(dn.getLhsBatchingDimensions())),
        b.getNamedAttr("rhs_batching_dimensions",
                       b.getDenseI64ArrayAttr(dn.getRhsBatchingDimensions())),
        b.getNamedAttr("lhs_contracting_dimensions",
                       b.getDenseI64ArrayAttr(dn.getLhsContractingDimensions())),
        b.getNamedAttr("rhs_contracting_dimensions",
                       b.getDenseI64ArrayAttr(dn.getRhsContractingDimensions())),
        b.getNamedAttr("algorithm", b.getI32IntegerAttr(0))};  // DS_DOT_TENSOR_INT8
    Value lhs = widen(b, loc, d.getLhs()), rhs = widen(b, loc, d.getRhs());
    replace(b, d, customCall(b, loc, "ds_dot_general_f64", withF64(d.getResult().getType()),
                             ValueRange{lhs, rhs}, cfg));
  }

  void rewriteReduce(OpBuilder& b, stablehlo::ReduceOp r) {
    Location loc = r.getLoc();
    SmallVector<NamedAttribute> cfg = {
        b.getNamedAttr("dimensions", b.getDenseI64ArrayAttr(r.getDimensions())),
        b.getNamedAttr("body", b.getI32IntegerAttr(*reduceBody(r)))};
    Value x = widen(b, loc, r.getInputs()[0]), init = widen(b, loc, r.getInitValues()[0]);
    replace(b, r, customCall(b, loc, "ds_reduce_f64", withF64(r.getResult(0).getType()),
                             ValueRange{x, init}, cfg));
  }

  void rewriteTree(OpBuilder& b, Operation* root, llvm::DenseSet<Operation*>& done) {
    Location loc = root->getLoc();
    const int32_t code = isa<stablehlo::AddOp>(root)        ? kAdd
                         : isa<stablehlo::SubtractOp>(root) ? kSub
                         : isa<stablehlo::MulOp>(root)      ? kMul
                                                            : kNeg;
    ProgramBuilder pb(b, loc, root->getBlock(), done);
    // The root's operands, absorbing the single-use trees below them; if
    // that exceeds ds_fused's limits, the root alone (its producers then
    // become programs of their own).  Converts made for a failed attempt are
    // unused and dropped at the end.
    Program p;
    bool fits = true;
    SmallVector<int32_t, 2> ids;
    for (Value v : root->getOperands()) {
      const int32_t id = pb.build(p, v, /*absorb=*/true);
      if (id < 0) fits = false;
      ids.push_back(id);
    }
    if (!fits) {
      p = Program();
      ids.clear();
      for (Value v : root->getOperands()) ids.push_back(pb.build(p, v, /*absorb=*/false));
    }
    p.push(code, ids[0], ids.size() > 1 ? ids[1] : 0, 0.0);
    SmallVector<NamedAttribute> cfg = {
        b.getNamedAttr("codes", b.getDenseI32ArrayAttr(p.codes)),
        b.getNamedAttr("a", b.getDenseI32ArrayAttr(p.a)),
        b.getNamedAttr("b", b.getDenseI32ArrayAttr(p.b)),
        b.getNamedAttr("values", b.getDenseF64ArrayAttr(p.values)),
        b.getNamedAttr("input_types", b.getDenseI32ArrayAttr(p.kinds)),
        b.getNamedAttr("out_type", b.getI32IntegerAttr(kKindF64))};
    Value call = customCall(b, loc, "ds_fused", withF64(root->getResult(0).getType()),
                            p.inputs, cfg);
    SmallVector<Operation*> absorbed(p.absorbed.begin(), p.absorbed.end());
    replace(b, root, call);
    for (Operation* op : llvm::reverse(absorbed)) {  // users before their operands
      done.insert(op);
      op->erase();
    }
  }

  // widen(narrow(x)) between two rewritten operations of one region is x
  // itself; then the marked converts nothing reads any more are dropped.
  void foldWidenedNarrowing(func::FuncOp func) {
    SmallVector<stablehlo::ConvertOp> widened;
    func.walk([&](stablehlo::ConvertOp c) {
      if (c->hasAttr(kWiden)) widened.push_back(c);
    });
    for (stablehlo::ConvertOp w : widened) {
      auto n = w.getOperand().getDefiningOp<stablehlo::ConvertOp>();
      if (n && n->hasAttr(kNarrow) && n->getParentRegion() == w->getParentRegion())
        w.getResult().replaceAllUsesWith(n.getOperand());
    }
    SmallVector<stablehlo::ConvertOp> marked;
    func.walk([&](stablehlo::ConvertOp c) {
      if (c->hasAttr(kWiden) || c->hasAttr(kNarrow)) marked.push_back(c);
    });
    for (stablehlo::ConvertOp c : llvm::reverse(marked))
      if (c.getResult().use_empty()) c->erase();
  }
};

}  // namespace

// Registers "ds-transform-b200" (for mlir-opt style tools and the plugin).
void registerDsTransformB200Pass() { PassRegistration<DsTransformB200Pass>(); }
