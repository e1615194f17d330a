"""A GPU session built from a checkpoint holds exactly the checkpoint's weights: its logits equal those of
a session built from the same parameters directly (ApplyCheckpointWeights, CheckpointReader.ts:71-73)."""
import json

import numpy as np
import pytest

from tests.helpers import O, pkg
from tests.test_checkpoint import _config

pytestmark = pytest.mark.gpu


def test_session_from_checkpoint_matches_direct_session(tmp_path):
    w = pkg.configs.MICROCHAT
    cfg = w.model
    p = pkg.init_params(cfg, 11)
    path = tmp_path / "microchat.ckpt"
    path.write_text(json.dumps(pkg.checkpoint.build_checkpoint(_config(cfg), p, cfg)))
    prompts = [O.uniform_ids(20, cfg.vocab_size, seed=40 + i) for i in range(3)]
    sess, cfg2 = pkg.checkpoint.session_from_checkpoint(str(path), max_seqs=3)
    assert cfg2 == cfg
    with sess, pkg.Session(cfg, p, max_seqs=3) as ref:
        for s in (sess, ref):
            s.prefill([0, 1, 2], [pr[:-1] for pr in prompts])
        a, _ = sess.step([0, 1, 2], [int(pr[-1]) for pr in prompts])
        b, _ = ref.step([0, 1, 2], [int(pr[-1]) for pr in prompts])
        assert np.array_equal(a, b)
