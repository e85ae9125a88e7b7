"""Host-side logic of the engine that needs no GPU: which component layouts one launch can cover, and the
``easyfhe.from_numpy`` tensor the reference's uploads go through."""
import numpy as np
import torch

from holmes_b200 import fhe as F


def test_component_runs():
    """Components stored one after another at one item stride form one run of comps x batch items (one launch);
    separate allocations, a different stride or a gap do not."""
    N, limbs, batch = 16, 3, 2
    storage = torch.zeros((2, batch, limbs + 1, N), dtype=torch.int64)
    cv = [storage[0], storage[1]]
    run = F._run(cv, batch)
    assert run is not None and run[1] == 2 * batch and run[2] == (limbs + 1) * N
    views = [c[:, :limbs] for c in cv]                # limb views keep the stride: still one run
    assert F._run(views, batch) is not None
    apart = [storage[0].clone(), storage[1].clone()]
    assert F._run(apart, batch) is None
    assert F._run([storage[0][:1], storage[1][:1]], 1) is None   # a gap of one item between the components
    (launch,) = F._runs(batch, cv, views)
    assert [t[1] for t in launch] == [2 * batch, 2 * batch]
    per_comp = F._runs(batch, cv, apart)
    assert len(per_comp) == 2 and all(t[1] == batch for launch in per_comp for t in launch)


def test_easyfhe_from_numpy_tensor():
    from holmes_b200 import easyfhe_compat as E

    a = np.arange(12, dtype=np.float64).reshape(3, 4)
    t = E.from_numpy(a)
    assert isinstance(t, torch.Tensor) and isinstance(t, E.HostTensor)
    np.testing.assert_array_equal(t.numpy(), a)
    assert type(t.to("cpu")) is torch.Tensor                     # host targets and dtype casts: plain Tensor.to
    np.testing.assert_array_equal(t.to(torch.float32).numpy(), a.astype(np.float32))
    np.testing.assert_array_equal(t.to(dtype=torch.int64).numpy(), a.astype(np.int64))


def test_bench_traffic_and_cpu_estimate():
    """The roofline line's traffic is the ncu capture's DRAM bytes scaled by algorithmic bytes (the capture's own
    launch gives back its measured bytes); the CPU estimate is the sum over families of bytes times seconds per byte,
    families without a sampled rate taking the key switch's."""
    import os

    import bench

    with open(os.path.join(bench.ROOT, "profiles", "traffic.txt"), encoding="utf-8") as f:
        family, measured, algorithmic = next(ln.split()[:3] for ln in f if ln.strip() and not ln.startswith("#"))
    assert bench.measured_traffic(family, int(algorithmic)) == int(measured)
    assert bench.measured_traffic(family, 2 * int(algorithmic)) == 2 * int(measured)
    assert bench.measured_traffic("no-such-family", 1) is None
    rates = {"rates_s_per_byte": {"keyswitch": 2e-9, "modup": 1e-9}}
    volume = {"keyswitch": {"bytes": 10}, "modup": {"bytes": 100}, "rescale": {"bytes": 5}}
    assert abs(bench.layer_cpu_estimate(volume, rates) - (10 * 2e-9 + 100 * 1e-9 + 5 * 2e-9)) < 1e-18
