"""Oracle-backed compute steps for zkie_b200.multigpu (TEST INFRASTRUCTURE).

Same methods as ``zkie_b200.multigpu.DeviceOps`` on CPU torch tensors, so the
split-commit orchestration (index math, all-to-all layout, collectives) runs
under gloo without a GPU.  The coset LDE is restated here from its definition
(row i of the LDE is X(W_H^i)): y[j'] = sum_m x[j' + m H/G] W_H^((j' + m H/G) g),
then the H/G-point DFT of y (oracle), and checked against the oracle's full
LDE by the tests.
"""
import numpy as np
import torch

P = 0xFFFFFFFF00000001


class OracleOps:
    def __init__(self, orc, consts):
        self.orc, self.consts = orc, consts

    @staticmethod
    def _np(t):
        return t.numpy() if isinstance(t, torch.Tensor) else np.asarray(t, dtype=np.uint64)

    def lde_coset(self, coeffs, lg_l, lg_b, w, lg_g, g):
        x = self._np(coeffs).reshape(1 << lg_l, w)
        lg_h = lg_l + lg_b
        H, G, L = 1 << lg_h, 1 << lg_g, 1 << lg_l
        R = H // G
        wh = self.orc.two_adic_generator(lg_h)
        y = np.zeros((R, w), dtype=object)
        for j in range(L):
            tw = pow(wh, (j * g) % H, P)
            y[j % R] = (y[j % R] + x[j].astype(object) * tw) % P
        out = self.orc.dft_batch(y.astype(np.uint64))
        return torch.from_numpy(np.ascontiguousarray(out).reshape(-1))

    def leaves(self, lde, rows, w):
        d = self.orc.merkle_leaves(self.consts, self._np(lde).reshape(rows, w))
        return torch.from_numpy(d.reshape(-1))

    def interleave(self, buf, G, n):
        a = self._np(buf).reshape(G, n, 8).transpose(1, 0, 2)
        return torch.from_numpy(np.ascontiguousarray(a).reshape(-1))

    def tree(self, leaves, n):
        root = self.orc.merkle_root_from_leaves(self.consts, self._np(leaves).reshape(n, 8))
        return None, torch.from_numpy(root.copy())


class OracleSumcheckOps:
    """Local degree-2 sumcheck by the oracle (sumcheck.rs:33-79 restated)."""

    def __init__(self, orc):
        self.orc = orc

    def sumcheck(self, f, h, challenges):
        f = f.numpy() if isinstance(f, torch.Tensor) else np.asarray(f, dtype=np.uint64)
        h = h.numpy() if isinstance(h, torch.Tensor) else np.asarray(h, dtype=np.uint64)
        rounds, finals = self.orc.sumcheck_prove(f, h, np.asarray(challenges, dtype=np.uint64))
        return np.asarray(rounds, dtype=np.uint64).reshape(-1, 3), int(finals[0]), int(finals[1])
