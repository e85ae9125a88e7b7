"""The tensor-core BSGS MAC (holmes_b200/csrc/mac_tc.cu, selected with HOLMES_MAC_TC=1) against the CUDA-core
kernel and exact integer arithmetic: identical residues for bench-like and ragged shapes (inputs and giants not multiples of 8,
babies not a multiple of 32), and its device error flag stays clear."""
import ctypes
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _run(monkeypatch, use_tc, ctx, out, c0s, c1s, bstride, nb, inputs, pts, pstride, G, limbs):
    from holmes_b200 import _lib as L
    if use_tc:
        monkeypatch.setenv("HOLMES_MAC_TC", "1")
    else:
        monkeypatch.delenv("HOLMES_MAC_TC", raising=False)
    L.call("holmes_bsgs_mac", ctx.handle, out.data_ptr(), c0s, c1s, bstride, nb, inputs, pts.data_ptr(), pstride, G,
           limbs, 0)


@pytest.mark.parametrize("inputs,G,nb,limbs", [(16, 8, 64, 3), (5, 3, 37, 2), (11, 9, 96, 1)])
def test_tc_mac_matches_cuda_core_and_oracle(monkeypatch, inputs, G, nb, limbs):
    import torch

    from holmes_b200 import _lib as L
    from holmes_b200 import fhe as F

    spec = F.CKKSContextSpec(depth=limbs + 2, log_n=12, dnum=2, dcrt_bits=59, first_mod=60, special_bits=60, seed=3,
                             auto_load_keys=False)
    client, ctx = F.generate_client_context(spec)
    try:
        N = ctx.N
        gen = torch.Generator(device="cuda").manual_seed(inputs * 100 + G)
        q = torch.tensor([ctx.q(i) for i in range(limbs)], dtype=torch.int64, device="cuda").view(1, limbs, 1)

        def rand(rows):
            r = torch.randint(0, 2 ** 62, (rows, limbs, N), device="cuda", dtype=torch.int64, generator=gen)
            return (r % q).to(torch.uint64)

        bab = rand(2 * nb * inputs).reshape(2, nb, inputs, limbs, N)
        pts = rand(G * nb)
        c0s = L.ptr_array([bab[0, :, i].data_ptr() for i in range(inputs)])
        c1s = L.ptr_array([bab[1, :, i].data_ptr() for i in range(inputs)])
        args = (c0s, c1s, inputs * limbs * N, nb, inputs, pts, limbs * N, G, limbs)
        out_tc = torch.empty((2, G, inputs, limbs, N), dtype=torch.uint64, device="cuda")
        out_cc = torch.empty_like(out_tc)
        _run(monkeypatch, True, ctx, out_tc, *args)
        _run(monkeypatch, False, ctx, out_cc, *args)
        torch.cuda.synchronize()
        flag = ctypes.c_int(1)
        L.call("holmes_device_error", 1, ctypes.byref(flag))
        assert flag.value == 0
        a, b = out_tc.cpu().numpy(), out_cc.cpu().numpy()
        np.testing.assert_array_equal(a, b)
        # one (component, giant, input, limb) row against exact integer arithmetic
        c, g, i, l = 1, G - 1, inputs - 1, limbs - 1
        qq = ctx.q(l)
        bb = bab[c, :, i, l].cpu().numpy().astype(object)
        pp = pts[g * nb:(g + 1) * nb, l].cpu().numpy().astype(object)
        want = np.array([int(v) % qq for v in (bb * pp).sum(axis=0)], dtype=np.uint64)
        np.testing.assert_array_equal(a[c, g, i, l], want)
    finally:
        ctx.close()
