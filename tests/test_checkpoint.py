"""Checkpoint loading: the reference's model.save / model.load
format (a pickled {state-dict name: array} dict, written by model.save at
flow2surf/training/optimization.py:41-42 and training/checkpoint.py:153,
read by predict.py:46) into Flow2SurfNet, on CPU."""

import collections
import os
import pickle

import numpy as np
import pytest

from flow2surf_b200 import build_model
from flow2surf_b200.params import parameter_specs
from flow2surf_b200.synthetic import random_parameters

TINY_CONFIG = {
    "k_neighbors": 8, "feat_dim": 32, "encoder_dims": [16, 24], "num_blocks": 2,
    "alpha_dim": 8, "ffn_ratio": 2, "decoder_dims": [16, 8],
}


def assert_same(model, params):
    got = model.state_dict()
    assert set(got) == set(params)
    for k, v in params.items():
        np.testing.assert_array_equal(got[k], np.asarray(v, dtype=np.float32))


def test_save_load_round_trip(tmp_path):
    params = random_parameters(TINY_CONFIG, seed=3)
    a = build_model(TINY_CONFIG)
    a.load_parameters(params)
    path = tmp_path / "model.pkl"
    a.save(path)
    b = build_model(TINY_CONFIG)
    b.load(path)
    assert_same(b, params)


@pytest.mark.parametrize("container", [dict, collections.OrderedDict])
def test_loads_a_pickled_state_dict(tmp_path, container):
    # what Jittor's Module.save writes: the state dict's Vars as NumPy arrays
    params = random_parameters(TINY_CONFIG, seed=4)
    path = tmp_path / "epoch_10.pkl"
    with open(path, "wb") as f:
        pickle.dump(container((k, np.asarray(v)) for k, v in params.items()), f)
    model = build_model(TINY_CONFIG)
    model.load(str(path))
    assert_same(model, params)


def test_loads_npz(tmp_path):
    params = random_parameters(TINY_CONFIG, seed=5)
    path = tmp_path / "weights.npz"
    np.savez(path, **params)
    model = build_model(TINY_CONFIG)
    model.load(path)
    assert_same(model, params)


class _Payload:
    def __reduce__(self):
        return (os.system, ("echo should-not-run",))


def test_refuses_code_in_a_checkpoint(tmp_path):
    path = tmp_path / "evil.pkl"
    with open(path, "wb") as f:
        pickle.dump({"x": _Payload()}, f)
    with pytest.raises(pickle.UnpicklingError):
        build_model(TINY_CONFIG).load(path)


def test_rejects_wrong_names_and_shapes(tmp_path):
    params = random_parameters(TINY_CONFIG, seed=6)
    name, shape, _ = parameter_specs(TINY_CONFIG)[0]
    bad = dict(params)
    bad[name] = np.zeros(tuple(s + 1 for s in shape), np.float32)
    path = tmp_path / "bad.pkl"
    with open(path, "wb") as f:
        pickle.dump(bad, f)
    with pytest.raises(ValueError):
        build_model(TINY_CONFIG).load(path)
    del bad[name]
    with open(path, "wb") as f:
        pickle.dump(bad, f)
    with pytest.raises(KeyError):
        build_model(TINY_CONFIG).load(path)
