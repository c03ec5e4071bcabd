"""The committed QWFIX001 fixtures under tests/golden/: the container layout
against the reference's own container test, and the CPU oracle against the
fixtures it wrote (any drift in the restatement changes their bits)."""

import os

import numpy as np
import pytest

from tests.golden import make_golden, qwfix


def test_container_layout_matches_reference_test():
    # fixture.zig:66-83: dims {2, 3}, six values, header then the f32 bits.
    values = np.array([1.0, -2.0, 3.5, 0.0, 1e-8, -1e8], np.float32)
    data = qwfix.encode([2, 3], values)
    assert len(data) == qwfix.HEADER_BYTES + 24
    assert data[:8] == b"QWFIX001"
    assert np.frombuffer(data[8:28], "<u4").tolist() == [2, 2, 3, 1, 1]
    assert np.array_equal(np.frombuffer(data[28:], "<u4"), values.view("<u4"))
    back = qwfix.decode(data)
    assert back.shape == (2, 3) and np.array_equal(back.ravel().view(np.uint32), values.view(np.uint32))


def test_container_errors():
    with pytest.raises(ValueError, match="RankTooLarge"):
        qwfix.encode([1, 1, 1, 1, 1], np.zeros(1, np.float32))
    with pytest.raises(ValueError, match="TooManyElements"):
        qwfix.encode([2, 3], np.zeros(5, np.float32))
    with pytest.raises(ValueError):
        qwfix.decode(b"QWFIX002" + bytes(20))
    with pytest.raises(ValueError):
        qwfix.decode(qwfix.encode([4], np.zeros(4, np.float32))[:-4])


@pytest.mark.parametrize("name", sorted(make_golden.FORMATS))
def test_fixture_ids_are_the_first_maximum_of_their_logits(name):
    tokens = qwfix.read(make_golden.path(name, "tokens"))
    logits = qwfix.read(make_golden.path(name, "logits"))
    assert logits.shape == (make_golden.STEPS + 1, make_golden.VOCAB)
    # decoder.zig:290-301: the first index of the maximum.
    assert [int(t) for t in tokens] == [int(np.argmax(row)) for row in logits]


@pytest.mark.parametrize("name", sorted(make_golden.FORMATS))
def test_oracle_reproduces_fixtures_bit_for_bit(oracle_lib, name):
    fresh = make_golden.generate(make_golden.FORMATS[name])
    for what, arr in fresh.items():
        stored = qwfix.read(make_golden.path(name, what))
        assert stored.shape == arr.shape, what
        assert np.array_equal(stored.view(np.uint32), arr.astype(np.float32).view(np.uint32)), what


def test_generator_is_committed_beside_fixtures():
    here = os.path.dirname(make_golden.__file__)
    names = sorted(f for f in os.listdir(here) if f.endswith(".qwfix"))
    assert names == sorted(f"decoder_{n}_{w}.qwfix" for n in make_golden.FORMATS
                           for w in ("tokens", "logits", "kv_last"))
