"""The decode prepack layout restatement (oracle/w4a8_oracle.py:stream_pack) is a permutation:
every code byte, scale and zero point of the op layout appears exactly once where the layout
says (checked on CPU by inverting it)."""
import numpy as np

import w4a8_oracle as O


def test_stream_pack_roundtrip():
    rng = np.random.default_rng(5)
    E, N, K = 2, 256, 1024
    w = rng.integers(-2 ** 31, 2 ** 31 - 1, (E, N, K // 8), dtype=np.int64).astype(np.int32)
    s = rng.uniform(1e-3, 2e-2, (E, N, K // 128)).astype(np.float16)
    z = rng.integers(-2 ** 31, 2 ** 31 - 1, (E, N // 8, K // 128), dtype=np.int64).astype(np.int32)
    for gate_up in (True, False):
        p = O.stream_pack(w, s, z, gate_up).reshape(E, -1, K // 512, O.PACK_BLOCK)
        nsl = p.shape[1]
        wb = w.view(np.uint8).reshape(E, N, K // 2)
        for e in range(E):
            for sl in range(nsl):
                for ch in range(K // 512):
                    blk = p[e, sl, ch]
                    for mm in (0, 5, 63, 64, 100, 127):
                        n = (sl * 64 + mm if mm < 64 else N // 2 + sl * 64 + mm - 64) if gate_up \
                            else sl * 128 + mm
                        for h in range(2):
                            for u in range(8):
                                got = blk[h * 16384 + mm * 128 + (u ^ (mm % 8)) * 16:][:16]
                                want = wb[e, n, ch * 256 + h * 128 + u * 16:][:16]
                                assert np.array_equal(got, want)
                        sc = blk[32768 + mm * 8:][:8].view(np.float16)
                        assert np.array_equal(sc, s[e, n, ch * 4:ch * 4 + 4])
                        if mm % 8 == 0:
                            zz = blk[33792 + (mm // 8) * 16:][:16].view(np.uint32)
                            assert np.array_equal(zz, z.view(np.uint32)[e, n // 8, ch * 4:ch * 4 + 4])
