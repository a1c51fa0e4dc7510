"""Split merges: the decode projection's k-segments and the decode attention's
position splits are merged inside thread-block clusters (distributed shared
memory) by default, or through global memory and arrival tickets with
MS_SPLITK_GLOBAL=1.  Both sum the same partials in the same order, so every
output -- projections, layer outputs, greedy ids -- must be bit-identical, and
repeated runs must agree (the merge order does not depend on timing)."""
import os
import subprocess
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))


def _run(tmp_path, name, global_merge):
    env = dict(os.environ)
    env.pop("MS_SPLITK_GLOBAL", None)
    if global_merge:
        env["MS_SPLITK_GLOBAL"] = "1"
    out = str(tmp_path / f"{name}.npz")
    subprocess.run([sys.executable, os.path.join(HERE, "split_merge_worker.py"), out],
                   env=env, check=True, timeout=600)
    return np.load(out)


@pytest.mark.gpu
def test_cluster_and_global_split_merges_are_bit_identical(tmp_path):
    a = _run(tmp_path, "cluster", False)
    b = _run(tmp_path, "global", True)
    c = _run(tmp_path, "cluster2", False)
    assert sorted(a.files) == sorted(b.files)
    for k in a.files:
        assert np.array_equal(a[k], b[k]), f"{k}: cluster and global merges differ"
        assert np.array_equal(a[k], c[k]), f"{k}: two cluster runs differ"
