"""CPU checks of the PoW-grinding oracle against a stateful pure-Python
DuplexChallenger (observe / sample / duplexing as the p3 duplex sponge)."""
import copy
import random

from tests import pyref
from tests.test_oracle import _consts_py

P = pyref.P


def states(cp, seed):
    """Challengers after mixed observe / sample sequences, with 0..7 inputs buffered."""
    rnd = random.Random(seed)
    out = []
    for buffered in range(8):
        ch = pyref.DuplexChallenger(cp)
        for _ in range(rnd.randrange(1, 12)):
            if rnd.random() < 0.6:
                ch.observe(rnd.randrange(P))
            else:
                ch.sample()
        ch.sample()  # no inputs buffered, some outputs left
        for _ in range(buffered):
            ch.observe(rnd.randrange(P))
        assert len(ch.inp) == buffered
        out.append(ch)
    return out


def test_check_witness_matches_stateful_challenger(orc, consts):
    cp = _consts_py(consts)
    rnd = random.Random(11)
    for ch in states(cp, 5):
        for bits in (0, 1, 3, 8):
            for _ in range(4):
                w = rnd.randrange(P)
                expect = copy.deepcopy(ch).check_witness(bits, w)
                assert orc.check_witness(consts, ch.state, ch.inp, bits, w) == expect


def test_grind_is_the_smallest_witness(orc, consts):
    cp = _consts_py(consts)
    for ch in states(cp, 9)[::3]:
        for bits in (2, 4):
            w = orc.grind(consts, ch.state, ch.inp, bits)
            assert copy.deepcopy(ch).check_witness(bits, w)
            assert not any(copy.deepcopy(ch).check_witness(bits, v) for v in range(w))
