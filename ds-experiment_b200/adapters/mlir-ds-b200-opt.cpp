//===- mlir-ds-b200-opt.cpp - opt driver for the retargeted DS pass ---------===//
//
// mlir-opt with the func and StableHLO dialects and the "ds-transform-b200"
// pass registered:
//
//   mlir-ds-b200-opt --ds-transform-b200 module.mlir
//
// The PJRT proxy (pjrt_plugin/ds_pjrt_plugin.cpp of the reference) runs its
// pass pipeline on each compiled module; pointing it at this pass makes the
// executable call libds_b200's targets (adapters/ds_b200_ffi.cc), which must
// be registered with XLA in the process before compile.
//
//===----------------------------------------------------------------------===//

#include "mlir/Dialect/Func/IR/FuncOps.h"
#include "mlir/IR/DialectRegistry.h"
#include "mlir/Tools/mlir-opt/MlirOptMain.h"
#include "stablehlo/dialect/Register.h"

void registerDsTransformB200Pass();

int main(int argc, char** argv) {
  registerDsTransformB200Pass();
  mlir::DialectRegistry registry;
  registry.insert<mlir::func::FuncDialect>();
  mlir::stablehlo::registerAllDialects(registry);
  return mlir::asMainReturnCode(
      mlir::MlirOptMain(argc, argv, "double-single transform (libds_b200 targets)", registry));
}
