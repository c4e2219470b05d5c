"""dp.MultiGPU on a real GPU: one spawned worker process on GPU 0 loads the model from a
picklable weights callable and transcribes the clips it is dealt; its lists equal
Bark.tokens_batch in this process."""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def two_layer_weights():
    from tinybark_b200 import synthetic, weights

    return weights.convert(synthetic.state_dict(0, layers=2), synthetic.config(2)), synthetic.config(2)


def test_multi_gpu_worker_matches_in_process_batch():
    import tinybark_b200
    from tinybark_b200 import synthetic
    from tinybark_b200.dp import MultiGPU

    rng = np.random.default_rng(12)
    clips = [synthetic.clip(float(s), 400 + i) for i, s in enumerate(rng.uniform(0.5, 12.0, 9))]
    with MultiGPU([0], weights=two_layer_weights) as m:
        got = m.tokens_batch(clips)
    want = tinybark_b200.load("gpu", weights=two_layer_weights()).tokens_batch(clips)
    assert got == want and sum(len(t) for t in got) > 0
