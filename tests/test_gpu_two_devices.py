"""Sessions on two devices in one process (the reference's backend handle lives for the process and its
entry points must be reentrant, Brain/ComputeBackend/GoFfiBackend.ts:36-42): kernel attributes and tensor
maps are set up per device, so a session on device 1 created after one on device 0 runs the same kernels
correctly. Independent sessions only: no peer memory, no multicast. Skipped with fewer than two GPUs."""
import numpy as np
import pytest

from tests.helpers import O, TOL_BF16, oracle_shape, pkg

pytestmark = pytest.mark.gpu


def _device_count() -> int:
    import torch
    return torch.cuda.device_count()


@pytest.mark.skipif("_device_count() < 2")
def test_sessions_on_two_devices_match_the_oracle():
    w = pkg.configs.MICROCHAT
    cfg = w.model
    params = pkg.init_params(cfg, w.weight_seed)
    model = O.Model(oracle_shape(cfg, "F32"), params.astype(np.float64))
    prompts = np.stack([O.uniform_ids(48, cfg.vocab_size, seed=2200 + i) for i in range(20)])
    outs = []
    for dev in (0, 1):
        with pkg.Session(cfg, params, max_seqs=20, device=dev) as sess:
            outs.append(sess.generate(prompts, 16))
            step_logits, _ = sess.step([0, 1], [3, 5])  # the per-kernel path on this device too
    for ids in outs:
        chk = model.check_trajectories(prompts, ids, TOL_BF16)
        assert int(chk["fails"].sum()) == 0
    assert np.array_equal(outs[0], outs[1])  # same build, same arithmetic on both devices
    assert pkg.load().ShahdDeviceErrorFlag() == 0
