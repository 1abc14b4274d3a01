"""Host-side checks of the StreamingLLM ring-cache format: the rows the
oracle's definition keeps are exactly the positions the last query can see
under the upstream token rule, and the Python class validates its inputs."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import streaming_oracle as orc


@pytest.mark.parametrize("sink,window,seq_len", [(4, 16, 1), (4, 16, 4), (4, 16, 20), (4, 16, 21),
                                                 (4, 16, 100), (0, 8, 50), (3, 0, 30),
                                                 (4, 2048, 100001)])
def test_ring_rows_hold_exactly_the_visible_positions(sink, window, seq_len):
    rows = orc.ring_cache_positions(sink, window, seq_len)
    held = set(int(p) for p in rows if p >= 0)
    qpos = seq_len - 1
    visible = {k for k in range(seq_len) if k < sink or qpos - k < window}
    assert held == visible
    if seq_len < 5000:
        tok = orc.streaming_token_mask(1, seq_len, sink, window)[0]
        assert visible == set(np.nonzero(tok)[0].tolist())


def test_cache_rejects_bad_geometry():
    from streaming_kv_cache import StreamingKVCache
    with pytest.raises(ValueError):
        StreamingKVCache(1, 1, 64, 0, 0)
    with pytest.raises(ValueError):
        StreamingKVCache(0, 1, 64, 4, 8)
    with pytest.raises(ValueError):
        StreamingKVCache(1, 1, 64, -1, 8)


def test_ring_abi_rejects_without_gpu():
    import sbfa_native as native
    lib = native.lib()
    assert lib.sbfa_ring_decode_workspace_bytes(64, 32, 128, 4, 2048) >= 0
    rc = lib.sbfa_ring_append(None, None, None, None, 1, 1, 64, 0, 4, 8, 0, 1, None)
    assert rc == 1 and "NULL" in native.last_error()
    rc = lib.sbfa_ring_decode(None, None, None, None, None, 1, 1, 64, 0, 1.0, 0, 0, 1, None, 0,
                              None)
    assert rc == 1 and "sink_size" in native.last_error()
    rc = lib.sbfa_ring_decode(None, None, None, None, None, 1, 1, 64, 3, 1.0, 4, 8, 1, None, 0,
                              None)
    assert rc == 2  # float64 has no ring-decode kernel
    _ = torch  # noqa
