"""Host side of sampling: the oracle's known answers from generation.rs's own
tests, and the seeded RNG chain of the Generator mirror (HKDF-SHA256 as
derive_seed uses it, adapteros-core/src/seed.rs:986-1016, checked against the
`cryptography` package's HKDF; ChaCha20 keystream word order checked against
RFC 7539 appendix A.1 test vector 1, which is also rand_chacha's zero-seed
output)."""
import numpy as np

from oracle import oracle as O
from tests.aos_import import aos


def test_oracle_known_answers():
    assert O.sample(np.array([0.1, 0.5, 0.3, 0.8, 0.2], np.float32), greedy=True)[0] == 3
    assert O.sample(np.array([1.0, 1.0, 0.5], np.float32), greedy=True)[0] == 1  # max_by keeps the later
    x = np.array([[1.0, 2.0, 3.0, 4.0, 5.0]], np.float32)
    assert O.sample(x, [0.999], top_k=1)[0] == 4
    assert O.sample(x, [0.0])[0] == 0
    assert O.sample(np.zeros((1, 4), np.float32), [0.3], top_k=0)[0] == 3  # degenerate -> argmax -> last


def test_hkdf_matches_reference_implementation():
    from cryptography.hazmat.primitives import hashes
    from cryptography.hazmat.primitives.kdf.hkdf import HKDF
    for ikm, info in ((bytes(32), b"sampling"), (bytes(range(32)), b"sample:7"), (b"\x0b" * 22, b"")):
        want = HKDF(algorithm=hashes.SHA256(), length=32, salt=None, info=info).derive(ikm)
        assert aos._hkdf_sha256(ikm, info) == want


def test_chacha_keystream_word_order():
    from cryptography.hazmat.primitives.ciphers import Cipher, algorithms
    enc = Cipher(algorithms.ChaCha20(bytes(32), bytes(16)), mode=None).encryptor()
    ks = enc.update(bytes(16))
    assert ks.hex() == "76b8e0ada0f13d90405d6ae55386bd28"
    assert int.from_bytes(ks[:4], "little") == 0xADE0B876


def test_rng_streams():
    a, b = aos.DeterministicRng(bytes(32), "sampling"), aos.DeterministicRng(bytes(32), "sampling")
    c = aos.DeterministicRng(bytes(32), "router")
    sa = [a.next_u32() for _ in range(100)]
    assert sa == [b.next_u32() for _ in range(100)]
    assert sa != [c.next_u32() for _ in range(100)]
    vals = [a.gen_f32() for _ in range(1000)]
    assert all(0.0 <= v < 1.0 for v in vals)
