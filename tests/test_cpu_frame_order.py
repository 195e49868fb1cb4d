"""The frame order of one video stream over several GPUs (csrc/frame_order.h, through
ajib_selftest_frame_order; host only): frame k goes to device k mod n and ring slot
(k / n) mod depth, a slot is reused only after its previous frame, and tickets count as finished
in submission order whatever order the devices finish them in (the order a one-device player
sees, the reference harness's loop, src/harness.c:646-700)."""
import numpy as np
import pytest

import ajib


@pytest.mark.parametrize("ndev,depth,n", [(1, 1, 5), (1, 3, 9), (2, 2, 11), (3, 2, 20), (8, 3, 100), (8, 1, 64)])
def test_places_and_in_order_completion(ndev, depth, n):
    rng = np.random.default_rng(ndev * 100 + depth)
    finish = rng.permutation(np.arange(1, n + 1))
    dev, slot, reuse, comp = ajib.frame_order(ndev, depth, finish)
    k = np.arange(n)
    assert np.array_equal(dev, k % ndev)
    assert np.array_equal(slot, (k // ndev) % depth)
    want_reuse = np.where(k >= ndev * depth, k - ndev * depth + 1, 0)
    assert np.array_equal(reuse, want_reuse)
    # completion: the longest prefix of finished tickets after each finish event
    done = np.zeros(n + 2, bool)
    c = 0
    for i, t in enumerate(finish):
        done[t] = True
        while done[c + 1]:
            c += 1
        assert comp[i] == c
    assert comp[-1] == n


def test_devices_finishing_out_of_order():
    """Device 1 finishes its frames first: nothing completes until device 0's first frame does."""
    dev, slot, reuse, comp = ajib.frame_order(2, 2, [2, 4, 1, 3])
    assert list(comp) == [0, 0, 2, 4]


def test_refuses_bad_arguments():
    assert ajib.lib.ajib_selftest_frame_order(0, 1, 0, None, None, None, None, None) == ajib.AJIB_ERR_ARGS
