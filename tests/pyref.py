"""Pure-Python restatement of the reference algorithms for small cases.

A second, independently written check of the C oracle (oracle/zkie_oracle.c):
slow big-int arithmetic, written straight from the reference sources cited
below, used only in tests on tiny inputs.
"""
P = 0xFFFFFFFF00000001


def inv(a):
    return pow(a, P - 2, P)


def two_adic_generator(bits):
    g = pow(7, (P - 1) >> 32, P)
    return pow(g, 1 << (32 - bits), P)


# ---- DFT (crates/zkie-core/cuda/goldilocks_ntt.cu:1-23 contract) ----------------------
def dft(col):
    n = len(col)
    lg = n.bit_length() - 1
    w = two_adic_generator(lg)
    return [sum(col[j] * pow(w, i * j, P) for j in range(n)) % P for i in range(n)]


# ---- Poseidon2 (crates/zkie-core/cuda/poseidon2_merkle.cu:37-155) ---------------------
def mat4(x):
    a, b, c, d = x
    return [(2 * a + 3 * b + c + d) % P, (a + 2 * b + 3 * c + d) % P,
            (a + b + 2 * c + 3 * d) % P, (3 * a + b + c + 2 * d) % P]


def mds_light(s):
    out = []
    for j in range(0, 16, 4):
        out += mat4(s[j:j + 4])
    sums = [sum(out[k + j] for j in range(0, 16, 4)) % P for k in range(4)]
    return [(out[i] + sums[i % 4]) % P for i in range(16)]


def diag(diag15):
    i2 = inv(2)
    return [P - 2, 1, 2, i2, 3, 4, P - i2, P - 3, P - 4, pow(i2, 3, P), pow(i2, 4, P), pow(i2, 5, P),
            P - pow(i2, 3, P), P - pow(i2, 4, P), P - pow(i2, 5, P), diag15]


def permute(state, ext_init, ext_final, internal, diag15):
    V = diag(diag15)
    s = [x % P for x in state]
    s = mds_light(s)
    for r in range(4):
        s = [pow((s[i] + ext_init[r][i]) % P, 7, P) for i in range(16)]
        s = mds_light(s)
    for r in range(22):
        s[0] = pow((s[0] + internal[r]) % P, 7, P)
        tot = sum(s) % P
        s = [(tot + V[i] * s[i]) % P for i in range(16)]
    for r in range(4):
        s = [pow((s[i] + ext_final[r][i]) % P, 7, P) for i in range(16)]
        s = mds_light(s)
    return s


def hash_row(row, consts):
    """PaddingFreeSponge<Perm,16,8,8> (overwrite mode)."""
    s = [0] * 16
    i = 0
    while i < len(row):
        chunk = row[i:i + 8]
        for j, x in enumerate(chunk):
            s[j] = x % P
        s = permute(s, *consts)
        i += 8
    return s[:8]


def compress(l, r, consts):
    return permute(list(l) + list(r), *consts)[:8]


def padded_len(raw, n=2):
    if raw <= 1:
        return raw
    if raw >= n:
        return -(-raw // n) * n
    return n


def merkle_root(rows, consts):
    layer = [hash_row(r, consts) for r in rows]
    layer += [[0] * 8] * (padded_len(len(layer)) - len(layer))
    while len(layer) > 1:
        raw = len(layer) // 2
        nxt = [compress(layer[2 * i], layer[2 * i + 1], consts) for i in range(raw)]
        nxt += [[0] * 8] * (padded_len(raw) - raw)
        layer = nxt
    return layer[0]


# ---- MLE / sumcheck (common/mle.rs, common/sumcheck.rs) ---------------------------
def mle_eval(vals, point):
    buf = [v % P for v in vals]
    for p in point:
        buf = [(buf[2 * i] + p * (buf[2 * i + 1] - buf[2 * i])) % P for i in range(len(buf) // 2)]
    return buf[0]


def sumcheck_prove(f, h, ch):
    f, h = list(f), list(h)
    rounds = []
    i2 = inv(2)
    for r in ch:
        y0 = sum(f[2 * s] * h[2 * s] for s in range(len(f) // 2)) % P
        y1 = sum(f[2 * s + 1] * h[2 * s + 1] for s in range(len(f) // 2)) % P
        y2 = sum((2 * f[2 * s + 1] - f[2 * s]) * (2 * h[2 * s + 1] - h[2 * s]) for s in range(len(f) // 2)) % P
        rounds.append((y0, (4 * y1 - y2 - 3 * y0) * i2 % P, (y2 - 2 * y1 + y0) * i2 % P))
        f = [(f[2 * s] + r * (f[2 * s + 1] - f[2 * s])) % P for s in range(len(f) // 2)]
        h = [(h[2 * s] + r * (h[2 * s + 1] - h[2 * s])) % P for s in range(len(h) // 2)]
    return rounds, f[0], h[0]


class DuplexChallenger:
    """DuplexChallenger<F, Perm, 16, 8> restated as a stateful object (the
    p3-challenger duplex sponge the WHIR transcript uses, pcs/whir.rs:42)."""

    def __init__(self, cp, state=None):
        self.cp = cp
        self.state = [x % P for x in (state if state is not None else [0] * 16)]
        self.inp, self.out = [], []

    def duplexing(self):
        for i, v in enumerate(self.inp):
            self.state[i] = v
        self.inp = []
        self.state = permute(self.state, *self.cp)
        self.out = self.state[:8]

    def observe(self, v):
        self.out = []
        self.inp.append(v % P)
        if len(self.inp) == 8:
            self.duplexing()

    def sample(self):
        if self.inp or not self.out:
            self.duplexing()
        return self.out.pop()

    def sample_bits(self, bits):
        return self.sample() & ((1 << bits) - 1)

    def check_witness(self, bits, w):
        self.observe(w)
        return self.sample_bits(bits) == 0
