"""The C-ABI library: it loads without a GPU, exports every entry point
include/prism_moe.h declares, and its structs have the header's layout."""
import ctypes as C
import re
from pathlib import Path

import pytest

from prism_inference_b200 import abi

HEADER = Path(__file__).resolve().parents[1] / "include" / "prism_moe.h"


@pytest.fixture(scope="module")
def lib():
    if not abi.LIB_PATH.exists():
        from prism_inference_b200 import build
        build.build()
    return abi.load()


def declared_functions():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(?:int|const char\*|void)\s+\**(prism_\w+)\s*\(", text)))


def test_header_declares_exactly_the_known_exports():
    assert declared_functions() == sorted(abi.EXPORTS)


def test_library_exports_every_declared_symbol(lib):
    for name in declared_functions():
        assert hasattr(lib, name), name


def _header_struct_fields(name):
    text = HEADER.read_text()
    m = re.search(r"typedef struct %s \{(.*?)\} %s;" % (name, name), text, re.S)
    body = re.sub(r"/\*.*?\*/", "", m.group(1), flags=re.S)
    fields = []
    for decl in body.split(";"):
        decl = decl.strip()
        if not decl:
            continue
        mm = re.match(r"(?:const\s+)?(\w+)\s*(\*?)\s*(.*)$", decl, re.S)
        fields += [f.strip() for f in mm.group(3).split(",")]
    return fields


@pytest.mark.parametrize("cname,pyt", [("prism_attn_params", abi.AttnParams),
                                       ("prism_router_params", abi.RouterParams),
                                       ("prism_expert_params", abi.ExpertParams),
                                       ("prism_proj_params", abi.ProjParams),
                                       ("prism_dense_params", abi.DenseParams),
                                       ("prism_block_desc", abi.BlockDesc),
                                       ("prism_stack_desc", abi.StackDesc)])
def test_struct_layout_matches_header(cname, pyt):
    assert [f for f, _ in pyt._fields_] == _header_struct_fields(cname)


def test_push_constant_blocks_match_the_shaders():
    """Field order = the GLSL push_constant declarations (13/8/10/5/17 int32)."""
    assert C.sizeof(abi.AttnParams) == 13 * 4
    assert C.sizeof(abi.RouterParams) == 8 * 4
    assert C.sizeof(abi.ExpertParams) == 10 * 4
    assert C.sizeof(abi.ProjParams) == 5 * 4
    assert C.sizeof(abi.DenseParams) == 17 * 4
    assert C.sizeof(abi.AttnParams) <= 128  # the reference's push-constant range (prism_moe_bench.cpp:113)


def test_no_gpu_is_an_error_not_a_crash(lib):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    h = C.c_void_p()
    rc = lib.prism_create(0, C.byref(h))
    assert rc != abi.PRISM_OK
    assert lib.prism_last_error_string()


def test_abi_version(lib):
    assert lib.prism_abi_version() == 1


def test_null_arguments_rejected(lib):
    rc = lib.prism_attn_window(None, None, None, 0, None, 0, None)
    assert rc == abi.PRISM_E_ARG
    assert b"NULL" in lib.prism_last_error_string()
    assert lib.prism_stack_forward(None, None, None, 1, None, None) == abi.PRISM_E_ARG


def test_null_handles_rejected_by_every_stack_call(lib):
    """Each stack entry point answers a NULL handle with PRISM_E_ARG (and a message) instead of
    touching it; none needs a GPU to do so."""
    f = C.c_float()
    t = C.c_int64()
    calls = {
        "prism_stack_status": lambda: lib.prism_stack_status(None, None),
        "prism_stack_inject_stall": lambda: lib.prism_stack_inject_stall(None, None),
        "prism_moe_block": lambda: lib.prism_moe_block(None, None, None, 1, None, None, None),
        "prism_stack_infer": lambda: lib.prism_stack_infer(None, None, None, 1, C.byref(f)),
        "prism_stack_submit": lambda: lib.prism_stack_submit(None, None, None, 1, None, C.byref(t)),
        "prism_stack_wait": lambda: lib.prism_stack_wait(None, 0, None),
        "prism_stack_profile": lambda: lib.prism_stack_profile(None, 1),
    }
    for name, call in calls.items():
        assert call() == abi.PRISM_E_ARG, name
        assert lib.prism_last_error_string(), name
    assert lib.prism_stack_destroy(None) == abi.PRISM_OK  # like free(NULL)
    assert lib.prism_stack_launch_count(None, 4) == 0
    assert lib.prism_stack_tokens_per_frame(None) == 0
