"""The allocation-free sort entry point, moe_sort_align_static_scratch.

It serves callers that cannot allocate device memory (a host framework that
owns all device allocations, or a serving process that forbids allocating
once running): the per-CTA histogram scratch lives in a fixed 256 KiB device
array inside the library instead of a caller workspace.  This test calls it
through the C ABI twice in a row and checks every output against the
workspace entry point moe_sort_align (integer outputs: bit-exact), and that
a request larger than the array is refused without a launch.  It sits in a
file of its own, collected last, and passes alone or after the other tests.
"""

import ctypes

import numpy as np
import pytest
import torch

from moe_inference_verify_microbench_b200 import _native, ops

pytestmark = pytest.mark.gpu


def _p(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _outputs(dev, R, e_local):
    mt = ops.max_tiles(R, e_local)
    return dict(
        counts=torch.full((e_local,), -7, dtype=torch.int32, device=dev),
        offsets=torch.full((e_local + 1,), -7, dtype=torch.int32, device=dev),
        offsets64=torch.full((e_local + 1,), -7, dtype=torch.int64, device=dev),
        perm=torch.full((max(R, 1),), -7, dtype=torch.int32, device=dev),
        inv=torch.full((max(R, 1),), -7, dtype=torch.int32, device=dev),
        tiles=torch.full((max(mt, 1), 4), -7, dtype=torch.int32, device=dev),
        num_tiles=torch.full((1,), -7, dtype=torch.int32, device=dev),
    ), mt


def _run(lib, ids, R, E, e_begin, e_local, ws=None):
    dev = ids.device
    o, mt = _outputs(dev, R, e_local)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    common = (_p(o["counts"]), _p(o["offsets"]), _p(o["offsets64"]), _p(o["perm"]), _p(o["inv"]),
              _p(o["tiles"]), mt, _p(o["num_tiles"]), _p(status), stream)
    if ws is None:
        rc = lib.moe_sort_align_static_scratch(_p(ids), R, E, e_begin, e_local, *common)
    else:
        rc = lib.moe_sort_align(_p(ids), R, E, e_begin, e_local, _p(ws), ws.numel(), *common)
    torch.cuda.synchronize(dev)
    assert rc == 0, _native.error_string(rc)
    assert int(status.item()) == 0
    return o


@pytest.mark.parametrize("R,E,e_begin,e_local", [(40000, 128, 0, 128), (131072, 128, 0, 128),
                                                 (9000, 64, 16, 32), (1, 16, 0, 16)])
def test_static_scratch_matches_workspace_entry_point(cuda, R, E, e_begin, e_local):
    lib = _native.load()
    rng = np.random.default_rng(R)
    ids = torch.from_numpy(rng.integers(0, E, size=R).astype(np.int32)).to(cuda)
    ws = torch.empty(lib.moe_sort_align_workspace_bytes(R, e_local), dtype=torch.uint8, device=cuda)
    ref = _run(lib, ids, R, E, e_begin, e_local, ws)
    nt = int(ref["num_tiles"].item())
    n = int(ref["offsets"][-1].item())
    for _ in range(2):  # two calls in a row share the same static scratch
        got = _run(lib, ids, R, E, e_begin, e_local)
        for key in ("counts", "offsets", "offsets64", "inv"):
            assert torch.equal(got[key][:R if key == "inv" else None], ref[key][:R if key == "inv" else None]), key
        assert torch.equal(got["perm"][:n], ref["perm"][:n])
        assert int(got["num_tiles"].item()) == nt
        assert torch.equal(got["tiles"][:nt], ref["tiles"][:nt])


def test_static_scratch_refuses_oversize(cuda):
    lib = _native.load()
    R, E = 4096 * 600, 128  # 1200 chunks of 2048 records x 128 experts > 65536 ints
    ids = torch.zeros(R, dtype=torch.int32, device=cuda)  # full size: in bounds either way
    o, mt = _outputs(cuda, R, E)
    rc = lib.moe_sort_align_static_scratch(_p(ids), R, E, 0, E, _p(o["counts"]), _p(o["offsets"]),
                                           None, _p(o["perm"]), None, _p(o["tiles"]), mt,
                                           _p(o["num_tiles"]), None,
                                           ctypes.c_void_p(torch.cuda.current_stream(cuda).cuda_stream))
    torch.cuda.synchronize(cuda)
    assert rc == -5  # MOE_RC_WORKSPACE: nothing launched
    assert int(o["counts"][0].item()) == -7
