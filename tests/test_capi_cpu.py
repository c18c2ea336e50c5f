"""C-ABI library checks that need no GPU: it loads, exports every symbol the
header declares, and rejects bad arguments before touching CUDA."""
import ctypes as C
import re
from pathlib import Path

import numpy as np
import pytest
import torch

import oracle
from trifuse_b200 import _lib
from trifuse_b200._lib import AffineWeight, MoeArgs, OLMoEConfig, lib

ROOT = Path(__file__).resolve().parent.parent


def declared_symbols():
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        text = h.read_text()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names |= set(re.findall(r"\b(tf_\w+)\s*\(", text))
    return sorted(names)


def test_library_exports_every_declared_symbol():
    L = lib()
    syms = declared_symbols()
    assert len(syms) >= 30
    missing = [s for s in syms if not hasattr(L, s)]
    assert not missing, missing
    # and the Python binding covers all of them with argtypes
    assert set(syms) <= set(_lib.SIGNATURES), set(syms) - set(_lib.SIGNATURES)


def test_abi_version_and_status_names():
    L = lib()
    assert L.tf_abi_version() == 1
    assert L.tf_status_name(7) == b"TF_ERR_CANCELLED"


def w(q=0x10, experts=0, out=64, inn=256, group=64, bits=4):
    return AffineWeight(q, 0x20, 0x30, experts, out, inn, group, bits)


def test_affine_validation_messages_mirror_reference():
    L = lib()
    bad = w(bits=3)
    assert L.tf_affine_qmm(C.c_void_p(0x100), 1, C.byref(bad), 1, C.c_void_p(0x200), None) == 1
    assert b"bits4/8 and group32/64/128" in L.tf_last_error()
    eight = w(bits=8)
    assert L.tf_affine_qmm(C.c_void_p(0x100), 1, C.byref(eight), 1, C.c_void_p(0x200), None) == 8
    odd = w(inn=100)
    assert L.tf_affine_qmm(C.c_void_p(0x100), 1, C.byref(odd), 1, C.c_void_p(0x200), None) == 2
    # stacked weight required for gather_qmm
    assert L.tf_affine_gather_qmm(C.c_void_p(0x100), 1, 1, None, C.c_void_p(0x300), 1, C.byref(w()), 0, 1,
                                  C.c_void_p(0x200), None) == 2
    # unaligned Q
    un = w(q=0x11)
    assert L.tf_affine_qmm(C.c_void_p(0x100), 1, C.byref(un), 1, C.c_void_p(0x200), None) == 1
    # unknown activation dtype
    assert L.tf_affine_qmm(C.c_void_p(0x100), 1, C.byref(w()), 7, C.c_void_p(0x200), None) == 1


def test_router_and_norm_validation():
    L = lib()
    assert L.tf_olmoe_route(C.c_void_p(0x100), 4, 65, 8, 1, C.c_void_p(0x200), C.c_void_p(0x300), None) == 2
    assert L.tf_olmoe_route(C.c_void_p(0x100), 4, 64, 0, 1, C.c_void_p(0x200), C.c_void_p(0x300), None) == 1
    assert L.tf_rms_norm(C.c_void_p(0x100), 2, 100, C.c_void_p(0x200), 1e-5, 1, C.c_void_p(0x300), None) == 2
    assert L.tf_rms_norm(C.c_void_p(0x100), 2, 256, C.c_void_p(0x200), 0.0, 1, C.c_void_p(0x300), None) == 1


def test_moe_geometry_validation():
    L = lib()
    a = MoeArgs()
    a.x = a.residual = a.out = 0x100
    a.tokens, a.hidden, a.intermediate, a.experts, a.top_k, a.act = 4, 256, 128, 8, 2, 1
    a.router.dense = 0x100
    a.gate_proj = w(experts=8, out=128, inn=256)
    a.up_proj = w(experts=8, out=128, inn=256)
    a.down_proj = w(experts=8, out=256, inn=128)
    nb = C.c_size_t()
    assert L.tf_moe_workspace_size(C.byref(a), C.byref(nb)) == 0 and nb.value > 0
    a.down_proj = w(experts=8, out=128, inn=256)
    assert L.tf_moe_workspace_size(C.byref(a), C.byref(nb)) == 2
    assert b"packed parameter geometry differs" in L.tf_last_error()


def test_route_count_and_workspace_limits():
    """order / inverse are int32: more than 2^31 - 1 routes is refused, and
    the expert hook refuses a NULL workspace even when its size is claimed."""
    L = lib()
    nb = C.c_size_t(1 << 40)
    p = C.c_void_p(0x100)
    assert L.tf_moe_route_sort(p, 1 << 28, 8, 64, p, p, p, p, nb.value, None) == 2
    assert b"bad geometry" in L.tf_last_error()
    a = MoeArgs()
    a.x = a.residual = a.out = 0x100
    a.tokens, a.hidden, a.intermediate, a.experts, a.top_k, a.act = 1 << 28, 256, 128, 8, 8, 1
    a.router.dense = 0x100
    a.gate_proj = w(experts=8, out=128, inn=256)
    a.up_proj = w(experts=8, out=128, inn=256)
    a.down_proj = w(experts=8, out=256, inn=128)
    assert L.tf_moe_workspace_size(C.byref(a), C.byref(nb)) == 2
    assert b"2^31 - 1 routes" in L.tf_last_error()
    g, u, d = w(experts=8, out=128, inn=256), w(experts=8, out=128, inn=256), w(experts=8, out=256, inn=128)
    assert L.tf_moe_expert_gpu(p, 4, 256, p, p, 2, 0, 128, 8, C.byref(g), C.byref(u), C.byref(d), 1, p, p,
                               None, 1 << 40, None) == 1
    assert b"NULL or unaligned" in L.tf_last_error()


C_HOST = r"""
#include <stdio.h>
#include <string.h>
#include "trifuse_b200.h"
int main(void) {
  if (tf_abi_version() != TF_ABI_VERSION) return 1;
  if (strcmp(tf_status_name(TF_ERR_CANCELLED), "TF_ERR_CANCELLED") != 0) return 2;
  tf_affine_weight w;
  memset(&w, 0, sizeof w);
  w.bits = 3; w.group_size = 64; w.out_features = 64; w.in_features = 256;
  if (tf_affine_qmm((void*)0x100, 1, &w, TF_DTYPE_F16, (void*)0x200, NULL) != TF_ERR_INVALID_ARGUMENT ||
      !strstr(tf_last_error(), "bits4/8")) return 3;
  size_t bytes = 0;
  if (tf_moe_route_sort_workspace_size(16, 8, 64, &bytes) != TF_OK || bytes == 0) return 4;
  puts("ok");
  return 0;
}
"""


def test_header_serves_a_plain_c_host(tmp_path):
    """A C99 host (what a cgo / FFI binding compiles against) builds with
    -pedantic -Werror against the header, links the library and gets the
    status codes and messages back without a GPU."""
    import shutil
    import subprocess
    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("gcc not available")
    src = tmp_path / "host.c"
    src.write_text(C_HOST)
    libdir = Path(_lib.LIB_PATH).resolve().parent
    exe = tmp_path / "host"
    subprocess.run([gcc, "-std=c99", "-Wall", "-Wextra", "-Werror", "-pedantic", f"-I{ROOT / 'include'}",
                    str(src), f"-L{libdir}", "-ltrifuse_b200", f"-Wl,-rpath,{libdir}", "-o", str(exe)],
                   check=True, capture_output=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert out.returncode == 0 and out.stdout.strip() == "ok", (out.returncode, out.stdout, out.stderr)


def test_model_config_admission():
    L = lib()
    h = C.c_void_p()
    bad = OLMoEConfig(2, 256, 2, 1, 128, 128, 512, 8, 2, 64, 1e-5, 10000.0, 1)  # GQA
    assert L.tf_model_create(C.byref(bad), 0, C.byref(h)) == 8
    bad = OLMoEConfig(2, 256, 2, 2, 128, 128, 512, 8, 9, 64, 1e-5, 10000.0, 1)  # top_k > experts
    assert L.tf_model_create(C.byref(bad), 0, C.byref(h)) == 2
    bad = OLMoEConfig(2, 256, 2, 2, 128, 128, 512, 8, 2, 64, 1e-5, 0.5, 1)  # theta <= 1
    assert L.tf_model_create(C.byref(bad), 0, C.byref(h)) == 1


def test_torch_quantizer_matches_oracle_bytes():
    from trifuse_b200.quant import affine_quantize
    rng = np.random.default_rng(9)
    w32 = oracle.round_bf16(rng.standard_normal((12, 512)).astype(np.float32) * 0.02)
    q0, s0, b0 = oracle.affine_quantize(w32)
    q1, s1, b1 = affine_quantize(torch.from_numpy(w32))
    assert np.array_equal(q1.numpy().astype(np.uint32), q0)
    assert np.array_equal(s1.numpy(), s0) and np.array_equal(b1.numpy(), b0)


def test_ops_refuse_cpu_tensors():
    from trifuse_b200 import ops
    x = torch.zeros(2, 64, dtype=torch.float16)
    with pytest.raises(ValueError):
        ops.native_olmoe_softmax(x)
