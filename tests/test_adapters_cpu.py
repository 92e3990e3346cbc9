"""The header-gated adapters (ds-experiment_b200/adapters/) agree with each
other and with the boundary, read as text: they cannot be compiled in this
image (no XLA-FFI or MLIR headers), so this keeps them from drifting.

- every XLA-FFI handler symbol the reference defines (cpp/*.cpp, cpp/*.cu)
  has a replacement in ds_b200_ffi.cc;
- every custom-call target the retargeted pass emits has a handler, and the
  attribute names the pass writes are the ones the handler binds;
- every C-ABI function the handlers call is declared in include/ds_b200.h.
"""
import os
import re

from conftest import ROOT

ADAPTERS = os.path.join(ROOT, "ds-experiment_b200", "adapters")
FFI = open(os.path.join(ADAPTERS, "ds_b200_ffi.cc")).read()
PASS = open(os.path.join(ADAPTERS, "DsTransformPassB200.cpp")).read()
HEADER = open(os.path.join(ROOT, "include", "ds_b200.h")).read()

REFERENCE_HANDLERS = ["DsFromF64", "DsToF64", "DsFromF32", "DsToF32", "DsAdd", "DsSub", "DsMul",
                      "DsFusedAddMul", "DsFusedAddMulToF64", "DsFusedAxpy",
                      "DsFusedAddMulToF64Cuda", "DsFusedAddSubToF64Cuda",
                      "DsRecurrenceAddMulToF64Cuda"]


def handler_symbols():
    direct = re.findall(r"XLA_FFI_DEFINE_HANDLER_SYMBOL\((\w+),", FFI)
    macro = re.findall(r"DS_(?:PACKED|CHAIN)_HANDLER\((\w+),", FFI)
    return set(direct) | set(macro)


def camel(target):
    return "".join(p[:1].upper() + p[1:] for p in target.split("_"))


def test_every_reference_handler_is_replaced():
    assert set(REFERENCE_HANDLERS) <= handler_symbols() - {"Symbol"}


def test_pass_targets_have_handlers_with_the_same_attributes():
    targets = set(re.findall(r'customCall\(b, loc, "(\w+)"', PASS))
    assert targets == {"ds_dot_general_f64", "ds_reduce_f64", "ds_fused"}
    symbols = handler_symbols()
    for t in targets:
        assert camel(t) in symbols, t
    written = set(re.findall(r'getNamedAttr\("(\w+)"', PASS))
    bound = set(re.findall(r'\.Attr<[^>]*>+\("(\w+)"\)', FFI))
    assert written <= bound, written - bound


def test_handlers_call_declared_entry_points():
    called = set(re.findall(r"\b(ds_[a-z0-9_]+)\(", FFI)) - {"ds_last_error"}
    declared = set(re.findall(r"DS_API\s+[\w\s\*]+?\b(ds_[a-z0-9_]+)\(", HEADER))
    assert called and called <= declared, called - declared


PROXY = open(os.path.join(ADAPTERS, "ds_pjrt_proxy_b200.cc")).read()


def test_pjrt_proxy_runs_the_retargeted_pass():
    """The proxy's default pipeline names the pass DsTransformPassB200.cpp
    registers, and the opt driver it spawns registers that pass."""
    name = re.search(r'getArgument\(\) const final \{ return "([\w-]+)"; \}', PASS).group(1)
    assert f"func.func({name})" in PROXY
    assert "mlir-ds-b200-opt" in PROXY
    driver = open(os.path.join(ADAPTERS, "mlir-ds-b200-opt.cpp")).read()
    assert "registerDsTransformB200Pass();" in driver


def test_pjrt_proxy_has_no_fixed_paths_or_leaked_buffers():
    """The reference's defects are gone: every temporary file comes from
    mkstemp, no pinned host buffer is allocated, and the plugin and tool
    paths are read from the environment; its flags keep their names."""
    assert not re.search(r'"/tmp/[\w.]+"', PROXY)
    assert "mkstemp" in PROXY and "cudaMallocHost" not in PROXY
    for var in ("DS_REAL_PLUGIN", "DS_OPT_BINARY", "DS_PASS_PIPELINE", "DS_BYPASS",
                "DS_TEST_PASSTHROUGH"):
        assert f'"{var}"' in PROXY, var
    # the rewritten program is released with its executable
    assert "PJRT_LoadedExecutable_Destroy = destroy_wrapper" in PROXY


def test_pass_guards_nested_regions():
    """Rewrites reach into control flow only: the region check admits while,
    if and case parents, every candidate goes through it, and a tree absorbs
    producers of its own block only."""
    guard = re.search(r"bool inRewritableRegion\(Operation\* op\) \{(.*?)\n\}", PASS, re.S).group(1)
    assert "stablehlo::WhileOp, stablehlo::IfOp, stablehlo::CaseOp" in guard
    assert "if (!op || !inRewritableRegion(op)) return false;" in PASS
    assert "def->getBlock() == block_" in PASS
