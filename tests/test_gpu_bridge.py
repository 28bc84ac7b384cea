"""Scheduler bridge round trips, as the reference checks them:
tests/unit/test_metadata_bridge.py (write_bridge then read_bridge_debug, every
field) and tests/integration/test_scheduler_bridge.py (read back by a kernel
through the bridge's device mapping)."""

import pytest
import torch

from adapterslotsplusplus_b200 import WarpPipeEngine

pytestmark = pytest.mark.gpu


def _write(engine, n, whittle, t_rem, gwar, lam, burst, promo, hot, tile, nseg, step, load):
    engine.write_bridge(torch.tensor(whittle, dtype=torch.float32), torch.tensor(t_rem, dtype=torch.float32),
                        torch.tensor(gwar, dtype=torch.float32), torch.tensor(lam, dtype=torch.float32),
                        torch.tensor(burst, dtype=torch.uint8), torch.tensor(promo, dtype=torch.uint8),
                        torch.tensor(hot, dtype=torch.uint8), torch.tensor(tile, dtype=torch.uint8), n, nseg, step,
                        load)


def test_bridge_fields_round_trip(cuda):
    engine = WarpPipeEngine()
    vals = dict(whittle=[0.1, 0.2, 0.3, 0.4, 0.5], t_rem=[1.0, 2.0, 3.0, 4.0, 5.0], gwar=[0.9, 0.8, 0.7, 0.6, 0.5],
                lam=[10.0, 20.0, 30.0, 40.0, 50.0], burst=[1, 0, 1, 0, 1], promo=[0, 1, 0, 1, 0], hot=[1, 1, 0, 0, 0],
                tile=[2, 1, 0, 2, 1])
    _write(engine, 5, **vals, nseg=3, step=42, load=0.75)
    d = engine.read_bridge_debug()
    close = lambda a, b: len(a) == len(b) and all(abs(x - y) < 1e-6 for x, y in zip(a, b))  # noqa: E731
    assert close(d["whittle_scores"], vals["whittle"])
    assert close(d["t_remaining_ms"], vals["t_rem"])
    assert close(d["gwar_pred_next3"], vals["gwar"])
    assert close(d["lambda_hat"], vals["lam"])
    assert d["burst_active"] == vals["burst"] and d["promo_eligible"] == vals["promo"]
    assert d["is_hot"] == vals["hot"] and d["tile_size_code"] == vals["tile"]
    assert d["num_active_adapters"] == 5 and d["num_segments"] == 3 and d["step_id"] == 42
    assert abs(d["global_load"] - 0.75) < 1e-6


def test_bridge_read_by_kernel(cuda):
    engine = WarpPipeEngine()
    n = 6
    whittle = [round(0.05 * i + 0.1, 4) for i in range(n)]
    _write(engine, n, whittle, [float(i) for i in range(n)], [1.0 - 0.1 * i for i in range(n)],
           [5.0 * i for i in range(n)], [i % 2 for i in range(n)], [1 - i % 2 for i in range(n)],
           [1 if i < 2 else 0 for i in range(n)], [i % 3 for i in range(n)], nseg=4, step=17, load=0.5)
    launches = engine.kernel_launches()
    r = engine.read_bridge_via_kernel()
    assert engine.kernel_launches() == launches + 1  # a kernel of this library read it
    assert max(abs(a - b) for a, b in zip(r[:n], whittle)) < 1e-6
    assert (int(r[n]), int(r[n + 1]), int(r[n + 2])) == (n, 4, 17)


def test_bridge_rejects_too_many_adapters(cuda):
    engine = WarpPipeEngine()
    z = [0.0] * 65
    with pytest.raises(RuntimeError, match="exceeds"):
        _write(engine, 65, z, z, z, z, [0] * 65, [0] * 65, [0] * 65, [0] * 65, nseg=0, step=0, load=0.0)
