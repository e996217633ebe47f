"""GPU parity of PoW grinding (zkie2_grind) with the oracle: the smallest
valid witness for challengers with 0..7 buffered inputs and 0..14 bits,
minimality at 20 bits and validity at 26."""
import pytest

from tests.test_grind_oracle import states
from tests.test_oracle import _consts_py

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("bits", [0, 1, 5, 10, 14])
def test_grind_matches_oracle(zk, orc, consts, bits):
    for ch in states(_consts_py(consts), 100 + bits):
        assert zk.grind(ch.state, ch.inp, bits) == orc.grind(consts, ch.state, ch.inp, bits)


def test_grind_minimal_at_20_bits_and_valid_at_26(zk, orc, consts):
    ch = states(_consts_py(consts), 7)[3]
    w = zk.grind(ch.state, ch.inp, 20)
    assert orc.check_witness(consts, ch.state, ch.inp, 20, w)
    assert orc.grind(consts, ch.state, ch.inp, 20, 0, w) is None  # nothing smaller
    w26 = zk.grind(ch.state, ch.inp, 26)
    assert orc.check_witness(consts, ch.state, ch.inp, 26, w26)


def test_grind_rejects_bad_arguments(zk):
    with pytest.raises(ValueError):
        zk.grind([0] * 16, [1] * 8, 4)
    with pytest.raises(zk.ZkieError):
        zk.grind([0] * 16, [], 63)
