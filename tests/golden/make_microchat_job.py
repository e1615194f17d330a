"""Writes tests/golden/microchat_job.json: the ids of the MicroChat decode job that bench.py times
(64 sequences, the bench's 128-id prompts, 384 greedy new ids), produced on a B200 by this build's
generate path, after every id of every sequence has passed the oracle's teacher-forced check.

    python tests/golden/make_microchat_job.py [out.json]

The checksum (sum of all ids) is the value bench.py prints as `output_checksums`; bench.py compares
its own run with this file. Run it again whenever a kernel change moves the arithmetic (an id may then
change at a near tie); it refuses to write a file for ids that fail the check.
"""
from __future__ import annotations

import hashlib
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402

from tests.helpers import O, TOL_BF16, oracle_shape, pkg  # noqa: E402


def job_ids() -> tuple[np.ndarray, np.ndarray]:
    w = pkg.configs.MICROCHAT
    cfg = w.model
    params = pkg.init_params(cfg, w.weight_seed)
    prompts = pkg.sharding.shard_prompts(w, 0)
    with pkg.Session(cfg, params, max_seqs=w.seqs) as sess:
        ids = sess.generate(prompts, w.new_tokens)
    return prompts, ids


def check(prompts: np.ndarray, ids: np.ndarray) -> dict:
    w = pkg.configs.MICROCHAT
    cfg = w.model
    params = pkg.init_params(cfg, w.weight_seed)
    model = O.Model(oracle_shape(cfg, "F32"), params.astype(np.float64))
    return model.check_trajectories(prompts, ids, TOL_BF16)


def summary(ids: np.ndarray) -> dict:
    return {"checksum": int(ids.astype(np.int64).sum()),
            "ids_sha256": hashlib.sha256(np.ascontiguousarray(ids, dtype=np.int32).tobytes()).hexdigest()}


def main() -> None:
    out = sys.argv[1] if len(sys.argv) > 1 else os.path.join(HERE, "microchat_job.json")
    prompts, ids = job_ids()
    chk = check(prompts, ids)
    bad = int(chk["fails"].sum())
    if bad:
        raise SystemExit(f"{bad} ids fail the oracle check (first sequence {int(np.argmax(chk['fails'] > 0))}); "
                         "no golden written")
    w = pkg.configs.MICROCHAT
    doc = {"workload": w.name, "seqs": w.seqs, "prompt_len": w.prompt_len, "new_tokens": w.new_tokens,
           **summary(ids), "near_ties": int(chk["near_ties"].sum()),
           "max_gap_of_range": float(chk["max_gap"].max()),
           "check": "every id of every sequence judged by the oracle teacher-forced on its own prefix "
                    "(argmax, or a near tie within 2e-2 of the logit range)"}
    with open(out, "w") as f:
        json.dump(doc, f, indent=1)
    print(json.dumps(doc))


if __name__ == "__main__":
    main()
