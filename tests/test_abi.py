"""CPU tests of the C-ABI boundary: the library loads without a GPU, exports
every symbol include/senmoe.h declares, its struct layouts match the ctypes
mirror, and host-side validation rejects bad arguments before any CUDA call."""
import ctypes as C
import os
import re
import subprocess
import tempfile

import pytest

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
HEADER = os.path.join(ROOT, "include", "senmoe.h")


def _declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(senmoe_\w+)\s*\(", src)))


@pytest.fixture(scope="module")
def senmoe():
    import build as b  # sen-mlx_b200/build.py (conftest puts sen-mlx_b200 on sys.path)
    b.build()
    import senmoe as s
    return s


def test_every_declared_symbol_is_exported(senmoe):
    L = C.CDLL(senmoe.LIB_PATH)
    declared = _declared_functions()
    assert len(declared) >= 9
    for name in declared:
        assert hasattr(L, name), f"{name} declared in senmoe.h but not exported"
    assert set(declared) == set(senmoe.SIGNATURES), "ctypes signature table out of sync with the header"


def test_struct_layouts_match_ctypes(senmoe):
    prog = r'''
#include <stdio.h>
#include <stddef.h>
#include "senmoe.h"
int main(void) {
  printf("%zu %zu %zu %zu %zu %zu %zu %zu\n", sizeof(SenMoeConfig), sizeof(SenMoeWeights), sizeof(SenMoeDebug),
         offsetof(SenMoeConfig, max_tokens), offsetof(SenMoeWeights, shared_gate_vector), sizeof(SenMoePeerInfo),
         offsetof(SenMoePeerInfo, arena_bytes), offsetof(SenMoePeerInfo, device));
  return 0;
}'''
    with tempfile.TemporaryDirectory() as d:
        c, exe = os.path.join(d, "t.c"), os.path.join(d, "t")
        open(c, "w").write(prog)
        subprocess.run(["gcc", "-I", os.path.join(ROOT, "include"), c, "-o", exe], check=True)
        out = subprocess.run([exe], capture_output=True, text=True, check=True).stdout.split()
    got = [int(v) for v in out]
    want = [C.sizeof(senmoe.SenMoeConfig), C.sizeof(senmoe.SenMoeWeights), C.sizeof(senmoe.SenMoeDebug),
            senmoe.SenMoeConfig.max_tokens.offset, senmoe.SenMoeWeights.shared_gate_vector.offset,
            C.sizeof(senmoe.SenMoePeerInfo), senmoe.SenMoePeerInfo.arena_bytes.offset,
            senmoe.SenMoePeerInfo.device.offset]
    assert got == want


def test_version_string(senmoe):
    assert senmoe.lib().senmoe_version().decode().startswith("senmoe 1")


def _cfg(senmoe, **kw):
    c = senmoe.SenMoeConfig()
    c.hidden_size, c.moe_intermediate_size, c.n_routed_experts, c.num_experts_per_tok = 2048, 768, 128, 8
    c.bits, c.group_size, c.norm_topk_prob, c.routed_scaling_factor = 4, 64, 1, 1.0
    c.max_tokens, c.expert_begin, c.expert_end = 64, 0, 128
    for k, v in kw.items():
        setattr(c, k, v)
    return c


@pytest.mark.parametrize("field,value,status", [
    ("bits", 3, 5), ("group_size", 32, 5), ("num_experts_per_tok", 0, 1), ("num_experts_per_tok", 200, 1),
    ("max_tokens", 0, 1), ("expert_end", 129, 1), ("hidden_size", 2004, 5), ("router_kind", 7, 5),
])
def test_layer_create_rejects_bad_config_on_host(senmoe, field, value, status):
    L = senmoe.lib()
    cfg = _cfg(senmoe, **{field: value})
    w = senmoe.SenMoeWeights()
    h = C.c_void_p()
    rc = L.senmoe_layer_create(C.byref(cfg), C.byref(w), 0, C.byref(h))
    assert rc == status, L.senmoe_last_error()
    assert L.senmoe_last_error().decode()
    assert not h.value


def test_layer_create_rejects_null_and_misaligned_weights(senmoe):
    L = senmoe.lib()
    cfg = _cfg(senmoe)
    w = senmoe.SenMoeWeights()
    h = C.c_void_p()
    assert L.senmoe_layer_create(C.byref(cfg), C.byref(w), 0, C.byref(h)) == senmoe.ERR_BAD_ARG
    for n in senmoe.WEIGHT_FIELDS[:10]:
        setattr(w, n, 0x10000)
    w.up_scales = 0x10008  # not 16-byte aligned
    assert L.senmoe_layer_create(C.byref(cfg), C.byref(w), 0, C.byref(h)) == senmoe.ERR_BAD_ARG
    assert "aligned" in L.senmoe_last_error().decode()


def test_gather_qmm_argument_checks(senmoe):
    L = senmoe.lib()
    # transpose=false is a form the reference never calls
    rc = L.senmoe_gather_qmm(None, 1, None, None, None, None, 1, 64, 32, 4, 0, 64, 4, 0, None, None)
    assert rc == senmoe.ERR_UNSUPPORTED
    rc = L.senmoe_gather_qmm(None, 1, None, None, None, None, 1, 64, 32, 4, 1, 64, 5, 0, None, None)
    assert rc == senmoe.ERR_UNSUPPORTED
    rc = L.senmoe_gather_qmm(None, 3, None, None, None, None, 4, 64, 32, 4, 1, 64, 4, 0, None, None)
    assert rc == senmoe.ERR_BAD_ARG  # 4 indices do not broadcast over 3 rows
    rc = L.senmoe_gather_qmm(None, 1, None, None, None, None, 0, 64, 32, 4, 1, 64, 4, 0, None, None)
    assert rc == senmoe.OK  # nothing to do


def test_forward_rejects_null_layer_and_bad_token_count(senmoe):
    L = senmoe.lib()
    assert L.senmoe_layer_forward(None, None, 1, None, None, None) == senmoe.ERR_BAD_ARG
    assert L.senmoe_layer_destroy(None) == senmoe.OK


def test_expert_parallel_entry_points_reject_null(senmoe):
    L = senmoe.lib()
    info = senmoe.SenMoePeerInfo()
    assert L.senmoe_layer_peer_info(None, C.byref(info)) == senmoe.ERR_BAD_ARG
    assert L.senmoe_layer_connect_peers(None, 0, 1, C.byref(info)) == senmoe.ERR_BAD_ARG
    assert b"NULL" in L.senmoe_last_error()


def test_python_gather_qmm_rejects_unsupported_broadcast(senmoe):
    import torch
    x = torch.zeros(2, 3, 1, 64, dtype=torch.bfloat16)
    w = torch.zeros(4, 32, 8, dtype=torch.int32)
    s = torch.zeros(4, 32, 1, dtype=torch.bfloat16)
    with pytest.raises(senmoe.SenMoeError):
        senmoe.gather_qmm(x, w, s, s, torch.zeros(5, 2, dtype=torch.int32))
    with pytest.raises(senmoe.SenMoeError):
        senmoe.gather_qmm(torch.zeros(2, 2, 64, dtype=torch.bfloat16), w, s, s, torch.zeros(2, dtype=torch.int32))
