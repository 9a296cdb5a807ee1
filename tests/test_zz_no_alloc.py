"""infernt_attention_decode_noalloc: the decode attention with its scratch
in a static device array instead of a caller workspace.

The GPU test runs it and infernt_attention_decode (same kernel, explicit
workspace) on identical inputs, two calls in a row (positions p and p + 1,
so the second call starts from the tickets the first one left), and asserts
the outputs and both caches are bit-identical.  The file name sorts last so
it also runs after every other GPU test in one session; it does not depend
on that order.  The oversize check needs no GPU."""
import numpy as np
import pytest

import infernt_b200 as ib


def rnd(n, seed):
    return np.random.default_rng(seed).standard_normal(n).astype(np.float32)


@pytest.mark.gpu
@pytest.mark.parametrize("nq,nkv,D,pos,splits", [
    (32, 4, 64, 287, 37),   # TinyLlama heads, 9 active splits
    (32, 8, 128, 1500, 18),  # Llama-3-8B heads, several tiles per split
    (8, 2, 64, 10, 1),       # one split: no merge
])
def test_noalloc_matches_workspace_entry_point(cuda, nq, nkv, D, pos, splits):
    ms = pos + 8
    qkv = [cuda.from_numpy(rnd(nq * D + 2 * nkv * D, 40 + i)).cuda() for i in range(2)]
    kc, vc = rnd(nkv * ms * D, 50), rnd(nkv * ms * D, 51)
    caches = {k: (cuda.from_numpy(kc).cuda(), cuda.from_numpy(vc).cuda()) for k in ("ws", "static")}
    outs = {k: cuda.zeros(nq * D, device="cuda") for k in caches}
    ws = cuda.zeros(ib.lib().infernt_attention_workspace_bytes(nq, nkv, D, splits), dtype=cuda.uint8,
                    device="cuda")
    for step in range(2):
        p = pos + step
        kd, vd = caches["ws"]
        ib.call("infernt_attention_decode", outs["ws"].data_ptr(), qkv[step].data_ptr(), kd.data_ptr(),
                vd.data_ptr(), nq, nkv, D, ms, p, 10000.0, splits, ws.data_ptr(), None)
        kd, vd = caches["static"]
        ib.call("infernt_attention_decode_noalloc", outs["static"].data_ptr(), qkv[step].data_ptr(),
                kd.data_ptr(), vd.data_ptr(), nq, nkv, D, ms, p, 10000.0, splits, None)
        cuda.cuda.synchronize()
        assert cuda.equal(outs["static"], outs["ws"]), step
        assert cuda.equal(caches["static"][0], caches["ws"][0]), step
        assert cuda.equal(caches["static"][1], caches["ws"][1]), step
        assert bool(cuda.isfinite(outs["static"]).all())


@pytest.mark.gpu
def test_noalloc_shapes_back_to_back(cuda):
    """Calls of different shapes in a row (4, then 8, then 2 KV heads, each
    many splits): each finds the tickets the previous shape left at zero and
    matches the workspace entry point."""
    for i, (nq, nkv, D, pos, splits) in enumerate([(32, 4, 64, 700, 37), (32, 8, 128, 900, 18),
                                                    (8, 2, 64, 333, 20)]):
        ms = pos + 4
        qkv = cuda.from_numpy(rnd(nq * D + 2 * nkv * D, 60 + i)).cuda()
        kc, vc = rnd(nkv * ms * D, 70 + i), rnd(nkv * ms * D, 80 + i)
        caches = {k: (cuda.from_numpy(kc).cuda(), cuda.from_numpy(vc).cuda()) for k in ("ws", "static")}
        outs = {k: cuda.zeros(nq * D, device="cuda") for k in caches}
        ws = cuda.zeros(ib.lib().infernt_attention_workspace_bytes(nq, nkv, D, splits), dtype=cuda.uint8,
                        device="cuda")
        kd, vd = caches["ws"]
        ib.call("infernt_attention_decode", outs["ws"].data_ptr(), qkv.data_ptr(), kd.data_ptr(), vd.data_ptr(),
                nq, nkv, D, ms, pos, 10000.0, splits, ws.data_ptr(), None)
        kd, vd = caches["static"]
        ib.call("infernt_attention_decode_noalloc", outs["static"].data_ptr(), qkv.data_ptr(), kd.data_ptr(),
                vd.data_ptr(), nq, nkv, D, ms, pos, 10000.0, splits, None)
        cuda.cuda.synchronize()
        assert cuda.equal(outs["static"], outs["ws"]), (nq, nkv, D)
        assert cuda.equal(caches["static"][0], caches["ws"][0]) and cuda.equal(caches["static"][1], caches["ws"][1])


def test_noalloc_rejects_oversize_scratch():
    """16 q heads per KV head, D = 128, 148 splits: 9.9 MB of partials,
    above the 512 KiB static scratch; rejected before any device work."""
    lib = ib.lib()
    assert lib.infernt_attention_workspace_bytes(128, 8, 128, 148) > 512 * 1024
    status = lib.infernt_attention_decode_noalloc(8, 8, 8, 8, 128, 8, 128, 16, 3, 1e4, 148, None)
    assert status == 1  # INFERNT_ERR_INVALID_ARGUMENT
    assert b"static scratch" in lib.infernt_last_error()
