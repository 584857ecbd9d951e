"""Failure detection on the device, without a GPU fault.

Every mbarrier wait in the kernels is bounded: after its limit it records an
error code in the per-device flag that ig_device_error() reads and lets the
kernel wind down, so a lost arrival ends as an error status, not a hung GPU.
The self-check entry point runs one such wait on a barrier that nothing
completes, with a 50 ms limit; the test checks that it gave up in about that
time, that the flag holds the timeout code until it is reset, and that the
device still computes correctly afterwards. Out-of-vocabulary ids given to
the device entry point are reported through the same flag, their rows read as
embedding row 0 (the host entry points refuse them before any work)."""
import ctypes as C

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_bounded_wait_gives_up_and_device_stays_usable(igdev, oracle_lib):
    from indecis_b200 import _capi, ops
    L = _capi.load()
    L.ig_device_error(1)
    timed_out, waited = C.c_int32(0), C.c_int64(0)
    _capi.check(L.ig_check_wait_timeout(50_000_000, C.byref(timed_out), C.byref(waited)))
    assert timed_out.value == 1
    assert 50_000_000 <= waited.value < 1_000_000_000, waited.value
    assert L.ig_device_error(1) == 1  # a TMA-stage wait gave up
    assert L.ig_device_error(0) == 0  # cleared
    # The same device still gives the oracle's bits.
    rng = np.random.default_rng(3)
    H, nh, D = 128, 2, 64
    lens = [40, 7]
    N = sum(lens)
    qkv = rng.standard_normal((N, 3 * H)).astype(np.float32)
    offs = np.array([0, 40, 47], np.int64)
    got = ops.attention(torch.from_numpy(qkv).cuda(), H, nh, offs, -1).cpu().numpy()
    want = np.zeros((N, H), np.float32)
    for s in range(2):
        a, b = offs[s], offs[s + 1]
        for h in range(nh):
            want[a:b, h * D:(h + 1) * D] = oracle_lib.attn8(qkv[a:b, h * D:(h + 1) * D],
                                                            qkv[a:b, H + h * D:H + (h + 1) * D],
                                                            qkv[a:b, 2 * H + h * D:2 * H + (h + 1) * D], -1,
                                                            np.float32(1 / np.sqrt(D)))
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_out_of_vocabulary_id_on_device_is_reported(igdev):
    from indecis_b200 import _capi
    from indecis_b200 import synthetic as S
    from indecis_b200.model import Config, Model
    cfg = S.tiny(layers=2, hidden=128, heads=2, intermediate=256, vocab=500)
    gm = Model.from_arrays(Config.from_dict(cfg), S.weights(cfg, seed=4))
    L = _capi.load()
    ids, offs = S.ids_fixed(3, 20, cfg["vocab"], seed=2)
    bad = ids.copy()
    bad[25] = 500
    L.ig_device_error(1)
    d_ids = torch.from_numpy(bad).cuda()
    out = torch.empty((3, cfg["hidden"]), dtype=torch.float32, device="cuda")
    _capi.check(L.ig_encode_device(gm._h, d_ids.data_ptr(), offs.ctypes.data, 3, _capi.IG_MODE_POOLED,
                                   out.data_ptr(), torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert L.ig_device_error(1) == 5
    zero = bad.copy()
    zero[25] = 0
    want = gm.EncodeSeqs((zero, offs))
    assert np.array_equal(out.cpu().numpy().view(np.uint32), want.view(np.uint32))
    assert L.ig_device_error(0) == 0
    gm.close()


def test_host_call_fails_while_a_wait_code_is_set(igdev, oracle_lib):
    """A host call copies the device error flag after its last kernel and
    fails while the flag holds a wait code (its results would not be valid);
    once the code is cleared, calls succeed with the oracle's bits."""
    import oracle
    from indecis_b200 import _capi
    from indecis_b200 import synthetic as S
    from indecis_b200.model import Config, Model
    cfg = S.tiny(layers=2, hidden=128, heads=2, intermediate=256, vocab=500)
    W = S.weights(cfg, seed=6)
    om, gm = oracle.Model(cfg, W), Model.from_arrays(Config.from_dict(cfg), W)
    ids, offs = S.ids_fixed(4, 30, cfg["vocab"], seed=5)
    want = om.encode(ids, offs)
    L = _capi.load()
    L.ig_device_error(1)
    assert np.array_equal(gm.EncodeSeqs((ids, offs)).view(np.uint32), want.view(np.uint32))
    timed_out = C.c_int32(0)
    _capi.check(L.ig_check_wait_timeout(20_000_000, C.byref(timed_out), None))
    assert timed_out.value == 1
    with pytest.raises(Exception, match="bounded wait"):
        gm.EncodeSeqs((ids, offs))
    assert L.ig_device_error(1) == 1
    assert np.array_equal(gm.EncodeSeqs((ids, offs)).view(np.uint32), want.view(np.uint32))
    gm.close()
