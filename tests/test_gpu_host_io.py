"""A step graph captured with its host traffic (StepFn.capture(host_io=True)):
the inputs copied from pinned staging buffers and the growth flags copied
back inside the graph. The steps must equal eager steps, and the pinned flags
must equal the device's.
"""

from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_host_io_graph_equals_eager_steps(cuda):
    import torch

    from plastax_b200 import StepInputs, make_step
    from plastax_b200.configs import ReservoirConfig, build_reservoir

    cfg = ReservoirConfig(num_units=1 << 12, fan_in=16, churn=0.01, capacity_align=256)
    xs = np.random.default_rng(9).standard_normal((8, cfg.num_inputs)).astype(np.float32)
    got = []
    for host_io in (False, True):
        net, static, state = build_reservoir(cfg, cuda)
        step = make_step(net, static, device=cuda)
        flags = []
        for i in range(len(xs)):
            if host_io and i == 3:
                step.capture(state, StepInputs(torch.from_numpy(xs[i]).to(cuda)), host_io=True)
            x = torch.from_numpy(xs[i])  # host inputs
            res = step(state, StepInputs(x if host_io else x.to(cuda)))
            torch.cuda.synchronize()
            if host_io and i >= 3:
                flags.append(step.host_flags.tolist())
                assert flags[-1] == [int(res.grown.item()), int(res.overflow.item())]
        assert int(state.grown.item()) > 0
        if host_io:
            assert all(g > 0 and o == 0 for g, o in flags)
        got.append({**{c: v.cpu().numpy() for c, v in state.conns[0].items()},
                    "activation": state.units["activation"].cpu().numpy()})
        step.close()
    for c in got[0]:
        np.testing.assert_array_equal(got[1][c], got[0][c], err_msg=c)
