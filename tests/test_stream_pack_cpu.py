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
                        n = ((N // 2 if mm % 2 else 0) + sl * 64 + mm // 2) if gate_up \
                            else sl * 128 + mm
                        for h in range(2):
                            for u in range(8):
                                got = blk[h * 16384 + mm * 128 + (u ^ (mm % 8)) * 16:][:16]
                                want = O.gemv_nibble_order(
                                    wb[e, n, ch * 256 + h * 128 + u * 16:][:16])
                                assert np.array_equal(got, want)
                        sc = blk[32768 + mm * 8:][:8].view(np.float16)
                        assert np.array_equal(sc, s[e, n, ch * 4:ch * 4 + 4])
                        zz = blk[33792 + (mm // 8) * 16:][:16].view(np.uint32)
                        nib = (zz >> np.uint32(4 * (mm % 8))) & 0xF
                        assert np.array_equal(nib, O.unpack_zeros(z, N)[e, n, ch * 4:ch * 4 + 4])


def test_gemv_nibble_order():
    """Word 0x76543210 (code i = i) becomes codes 0 2 4 6 1 3 5 7."""
    b = np.array([0x76543210], "<u4").view(np.uint8)
    assert O.gemv_nibble_order(b).view("<u4")[0] == 0x75316420
