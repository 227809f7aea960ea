"""``jaxml_b200.utils`` (the reference's ``jaxml.utils`` helpers) on CPU."""
import logging

import numpy as np
import pytest
import torch

from jaxml_b200 import utils


def test_reexports():
    from jaxml_b200.cache import get_default_pos_ids
    from jaxml_b200.hf_utils import torch_to_jax_states

    assert utils.get_default_pos_ids is get_default_pos_ids and utils.torch_to_jax_states is torch_to_jax_states
    mask = torch.tensor([[True, True, True, False, False], [True, False, False, False, False]])
    assert utils.get_default_pos_ids(mask).tolist() == [[2], [0]]


def test_check_shape():
    x = torch.zeros(2, 3, 4)
    utils.check_shape(x, 2, 3, 4)
    utils.check_shape(x, (2, None, 4))
    utils.check_shape(x, ..., 4)
    utils.check_shape(x, 2, ...)
    for bad in ((2, 3), (2, 3, 5), (None, 4), (..., 3)):
        with pytest.raises(AssertionError):
            utils.check_shape(x, *bad)


def test_pprint_pytree_and_timeit(capsys, caplog):
    utils.pprint_pytree({"a": torch.zeros(2, 3), "b": [np.ones(4, dtype=np.float32), 3]})
    out = capsys.readouterr().out
    assert "<Array shape=(2, 3) dtype=torch.float32>" in out and "<Array shape=(4,) dtype=float32>" in out
    log = logging.getLogger("jaxml_b200.test_timeit")

    @utils.timeit(log)
    def add(a, b):
        return a + b

    with caplog.at_level(logging.INFO, logger="jaxml_b200.test_timeit"):
        assert add(1, 2) == 3
        assert add(1, 2, log=False) == 3
    assert sum("Execution time for add" in r.message for r in caplog.records) == 1
