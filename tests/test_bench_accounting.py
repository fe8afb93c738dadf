"""The roofline arithmetic of bench.py, checked on the CPU by direct sums:
the K/V bytes a request's forward steps read and append (the decode's
algorithmic bytes beside the weight stream) and the useful flops of a codec
decode (its denominator-free achieved rate)."""
import importlib
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _bench():
    sys.path.insert(0, ROOT)
    return importlib.import_module("bench")


def test_kv_bytes_closed_form_equals_the_step_sum():
    b = _bench()
    for layers, rows, steps in ((24, 235, 1023), (2, 7, 40), (24, 451, 127), (1, 1, 1)):
        # forward step i attends over rows + i cached keys and appends one more
        direct = sum(b.KV_ROW_BYTES * layers * ((rows + i) + 1) for i in range(steps))
        assert b.kv_read_bytes(layers, rows, steps) == direct


def test_codec_flops_equal_the_layer_sum():
    b = _bench()
    D, F, H = 384, 2048, 1024
    for T in (1, 17, 300, 1024):
        gemms = [(T, D, H * 7)]                                  # embed conv k7 1024 -> 384
        gemms += [(T, F, D), (T, D, F)] * 12                     # pwconv1, pwconv2
        gemms += [(T, H, D), (2 * T, H, H * 3)]                  # head linear, up conv k3 over 2T rows
        direct = sum(2 * m * n * k for m, n, k in gemms) + 12 * 2 * T * D * 7  # + depthwise convs
        assert b.codec_flops(T) == direct
    assert b.codec_flops(1024) == 58048118784  # the figure in the committed codec bench line
