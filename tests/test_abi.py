"""C-ABI boundary on the CPU: the library loads, exports every symbol that
include/turboadam_b200.h declares, struct layouts agree with the header, and
host-side validation rejects bad input without touching a GPU."""
import ctypes
import os
import re

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "turboadam_b200.h")


@pytest.fixture(scope="module")
def lib():
    from turboadam_b200 import _lib
    from turboadam_b200.csrc import build

    build.build(quiet=True)
    return _lib.load()


def declared_symbols():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"TA_API\s+[\w\s\*]+?\b(ta_\w+)\s*\(", src)))


def test_header_symbols_exported(lib):
    from turboadam_b200 import _lib

    names = declared_symbols()
    assert len(names) == 22
    assert sorted(_lib.EXPORTED) == names
    for n in names:
        assert hasattr(lib, n), n
    assert lib.ta_abi_version() == 4


def test_struct_layout_matches_header(lib):
    from turboadam_b200 import _lib

    # compile a tiny C program against the header and compare offsets
    import subprocess
    import tempfile

    prog = r"""
#include <stdio.h>
#include <stddef.h>
#include "turboadam_b200.h"
int main(void) {
  printf("%zu %zu %zu %zu %zu %zu %zu\n", sizeof(ta_tensor), offsetof(ta_tensor, v_idx_dev),
         offsetof(ta_tensor, v_out_dev), sizeof(ta_group), offsetof(ta_group, bc1),
         offsetof(ta_group, v_bits), offsetof(ta_tensor, global_blocks));
  return 0;
}
"""
    with tempfile.TemporaryDirectory() as d:
        c = os.path.join(d, "t.c")
        exe = os.path.join(d, "t")
        open(c, "w").write(prog)
        subprocess.check_call(["gcc", "-I", os.path.dirname(HEADER), c, "-o", exe])
        got = [int(x) for x in subprocess.check_output([exe]).split()]
    want = [ctypes.sizeof(_lib.TaTensor), _lib.TaTensor.v_idx_dev.offset,
            _lib.TaTensor.v_out_dev.offset, ctypes.sizeof(_lib.TaGroup), _lib.TaGroup.bc1.offset,
            _lib.TaGroup.v_bits.offset, _lib.TaTensor.global_blocks.offset]
    assert got == want
    assert _lib.TENSOR_DTYPE.itemsize == want[0]


def test_padded_blocks_and_workspace(lib):
    from turboadam_b200 import _lib

    assert lib.ta_state_padded_blocks(1, 128) == 16
    assert lib.ta_state_padded_blocks(2048, 128) == 16
    assert lib.ta_state_padded_blocks(2049, 128) == 32
    arr = np.zeros(2, dtype=_lib.TENSOR_DTYPE)
    arr["numel"] = [5000, 100]
    arr["flags"] = [_lib.TA_M_COSTATE | _lib.TA_V_ONEQ, _lib.TA_V_ONEQ]
    ws = lib.ta_workspace_size(arr.ctypes.data, 2)
    assert ws > 3 * 2 * 2048 * 4


def _one_tensor(**over):
    from turboadam_b200 import _lib

    arr = np.zeros(1, dtype=_lib.TENSOR_DTYPE)
    r = arr[0]
    r["param_dev"] = 4096
    r["grad_dev"] = 8192
    r["numel"] = 1000
    r["flags"] = _lib.TA_V_ONEQ
    r["v_idx_dev"] = 16384
    r["v_hdr_dev"] = 32768
    r["exp_avg_dev"] = 65536
    r["step"] = 1
    for k, v in over.items():
        r[k] = v
    g = np.zeros(1, dtype=_lib.GROUP_DTYPE)
    g[0]["block_size"] = 128
    g[0]["v_bits"] = 4
    g[0]["bc1"] = g[0]["bc2"] = 1.0
    return arr, g


@pytest.mark.parametrize(
    "over,group_over,code",
    [
        ({"dtype": 7}, {}, 1),
        ({"group": 3}, {}, 1),
        ({}, {"v_bits": 5}, 1),
        ({}, {"block_size": 64}, 3),
        ({"step": 0}, {}, 1),
        ({"grad_dev": 0}, {}, 1),
        ({"param_dev": 4100}, {}, 2),
        ({"exp_avg_dev": 0}, {}, 1),
    ],
)
def test_validation_errors(lib, over, group_over, code):
    arr, g = _one_tensor(**over)
    for k, v in group_over.items():
        g[0][k] = v
    rc = lib.ta_step(arr.ctypes.data, 1, g.ctypes.data, 1, 0, 1 << 20, 1 << 30, None)
    assert rc == code, lib.ta_last_error()
    assert lib.ta_last_error()


def test_optimizer_constructor_api():
    import torch

    from turboadam_b200 import TurboAdam

    p = [torch.nn.Parameter(torch.randn(10, 10))]
    opt = TurboAdam(p, lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=1e-2)
    assert opt.defaults["weight_decay"] == 1e-2
    d = TurboAdam(p).defaults
    assert (d["lr"], d["betas"], d["eps"], d["weight_decay"], d["block_size"], d["v_bits"],
            d["compress_m"], d["compress_v"]) == (1e-3, (0.9, 0.999), 1e-8, 0.0, 128, 4, True, True)
    assert TurboAdam(p, block_size=64, v_bits=6).defaults["v_bits"] == 6
    with pytest.raises(ValueError, match="v_bits must be one of"):
        TurboAdam(p, v_bits=10)
    # capturable=True, which the reference refuses, is built here
    assert TurboAdam(p, capturable=True)._capturable
    assert TurboAdam._step_supports_amp_scaling


def test_cpu_params_fail_loudly():
    """No CPU fallback: a step on CPU tensors raises."""
    import torch

    from turboadam_b200 import TurboAdam
    from turboadam_b200._lib import TurboAdamBackendError

    p = torch.nn.Parameter(torch.randn(10))
    opt = TurboAdam([p])
    p.grad = torch.randn(10)
    with pytest.raises(TurboAdamBackendError):
        opt.step()
