"""Device-sampler host pieces on the CPU: the Philox-4x32-10 generator against the published known-answer
vectors of its authors (Random123), the parameter-block layout, per-request seeds."""
import numpy as np
import pytest

from fak_b200.engine.sampling import SamplingParams, pack_params, request_seed


def _ext():
    try:
        import torch  # noqa: F401  (the extension links against torch's libraries)
        from fak_b200.ops._ext import ext
        return ext()
    except ImportError:
        pytest.skip("extension not built")


@pytest.mark.parametrize("ctr,key,want", [
    ([0, 0, 0, 0], [0, 0], [0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8]),
    ([0xFFFFFFFF] * 4, [0xFFFFFFFF] * 2, [0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD]),
    ([0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344], [0xA4093822, 0x299F31D0],
     [0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1]),
])
def test_philox_known_answers(ctr, key, want):
    got = _ext().philox4x32_10_host(ctr, key).tolist()
    assert got == want, [hex(x) for x in got]


def test_pack_params_layout():
    sps = [SamplingParams(temperature=0.7, top_k=40, top_p=0.9, frequency_penalty=0.5, presence_penalty=0.25,
                          logit_bias={7: 3.0, 2: -1.0}),
           SamplingParams(), SamplingParams(temperature=1.0, logit_bias={9: 100.0})]
    P, tok, val = pack_params(sps, [3, 0, 11], [0x1122334455667788, 5, (1 << 64) - 1])
    f = P.view(np.float32)
    assert P.shape == (3, 10) and P.dtype == np.int32
    assert np.isclose(f[0, 0], 0.7) and P[0, 1] == 40 and np.isclose(f[0, 2], 0.9)
    assert np.isclose(f[0, 3], 0.5) and np.isclose(f[0, 4], 0.25)
    assert (P[0, 5], P[0, 6]) == (0, 2) and (P[2, 5], P[2, 6]) == (2, 1)
    assert tok.tolist() == [2, 7, 9] and val.tolist() == [-1.0, 3.0, 100.0]       # sorted per row
    assert P[0, 7].view(np.uint32) == 0x55667788 and P[0, 8].view(np.uint32) == 0x11223344
    assert P[2, 7] == -1 and P[2, 8] == -1 and P[2, 9] == 11


def test_request_seeds_are_distinct_and_stable():
    s = [request_seed(0, i) for i in range(1000)]
    assert len(set(s)) == 1000 and all(0 <= x < 1 << 64 for x in s)
    assert s == [request_seed(0, i) for i in range(1000)] and request_seed(1, 0) != s[0]
