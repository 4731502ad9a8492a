"""The tuning sweep's candidate entries (no GPU: the library's host-side
launch checks only)."""
import pytest

from dsa_b200 import api, config, tune


@pytest.mark.parametrize("name", sorted(config.CASE_SHAPES))
def test_candidates_are_valid_entries(name):
    shape = config.CASE_SHAPES[name]
    cands = tune.candidates(shape)
    assert cands and all(isinstance(t, config.Tuning) for t in cands)
    accepted = 0
    for t in cands:
        try:
            api._check_tuning(t, shape, 28)
            api._launch_from_tuning(t, shape)
            accepted += 1
        except ValueError:
            pass  # an entry the shape does not support (e.g. a union launch with SQ % (128 / H) != 0)
    assert accepted >= 2, name


def test_selected_entries_resolve():
    for name, t in config.SELECTED.items():
        assert config.select(config.CASE_SHAPES[name]) == t
