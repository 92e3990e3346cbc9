//===- mlir-ds-b200-opt.cpp - opt driver for the retargeted DS pass ---------===//
//
// mlir-opt with the func and StableHLO dialects, StableHLO's passes (the
// VHLO version conversions a PJRT program needs) and the "ds-transform-b200"
// pass registered:
//
//   mlir-ds-b200-opt --ds-transform-b200 module.mlir
//
// The PJRT proxy (adapters/ds_pjrt_proxy_b200.cc, after the reference's
// pjrt_plugin/ds_pjrt_plugin.cpp) runs its pipeline on each compiled
// module; this pass makes the executable call libds_b200's targets
// (adapters/ds_b200_ffi.cc), which must be registered with XLA in the
// process before compile.
//
//===----------------------------------------------------------------------===//

#include "mlir/Dialect/Func/IR/FuncOps.h"
#include "mlir/IR/DialectRegistry.h"
#include "mlir/Tools/mlir-opt/MlirOptMain.h"
#include "stablehlo/dialect/Register.h"
#include "stablehlo/transforms/Passes.h"

void registerDsTransformB200Pass();

int main(int argc, char** argv) {
  registerDsTransformB200Pass();
  mlir::stablehlo::registerPasses();
  mlir::DialectRegistry registry;
  registry.insert<mlir::func::FuncDialect>();
  mlir::stablehlo::registerAllDialects(registry);
  return mlir::asMainReturnCode(
      mlir::MlirOptMain(argc, argv, "double-single transform (libds_b200 targets)", registry));
}
