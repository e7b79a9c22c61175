"""The `.weights` format on the CPU (parser.zig:446-591): the byte layout of a save, the
round trip, the legacy header with a 32-bit `seen`, pre-2015 transposed connected weights,
`flipped` conv weights, the dontload / dontsave / dontloadscales flags, and the C++ host's
copy of the format (darknet_zig_b200/host/weights.hpp) agreeing byte for byte."""
from __future__ import annotations

import os
import struct
import subprocess
import sys

import numpy as np
import pytest

from darknet_zig_b200 import synth
from darknet_zig_b200.weights import LayerParams, load, save

NAMES = ("biases", "scales", "rolling_mean", "rolling_variance", "weights")


def network(seed: int = 0) -> list[LayerParams]:
    """conv+BN (8 filters, 3x3 over 4 channels), connected+BN (12 -> 5), standalone BN (6),
    conv without BN (3 filters, 1x1 over 8). tests/cpp/weights_rt.cpp builds the same."""
    layers = [
        LayerParams("convolutional", n=8, batch_normalize=True, nweights=8 * 4 * 3 * 3),
        LayerParams("connected", n=5, batch_normalize=True, inputs=12),
        LayerParams("batchnorm", n=6),
        LayerParams("convolutional", n=3, nweights=3 * 8),
    ]
    k = 0
    for layer in layers:
        for name in NAMES:
            a = getattr(layer, name)
            if a is not None:
                a[...] = synth.normal(900 + seed * 50 + k, (a.size,), 0.0, 1.0)
                k += 1
    return layers


def blank(layers):
    return [LayerParams(l.kind, n=l.n, batch_normalize=l.batch_normalize, nweights=l.nweights, inputs=l.inputs)
            for l in layers]


def test_save_writes_the_reference_layout(tmp_path):
    net = network()
    path = str(tmp_path / "a.weights")
    save(path, net, seen=123456789012)
    c, f, b, s = net
    want = struct.pack("<iiiQ", 0, 2, 0, 123456789012)
    for a in (c.biases, c.scales, c.rolling_mean, c.rolling_variance, c.weights,  # parser.zig:535-543
              f.biases, f.weights, f.scales, f.rolling_mean, f.rolling_variance,  # :545-553
              b.scales, b.rolling_mean, b.rolling_variance,                       # :555-559
              s.biases, s.weights):
        want += a.astype("<f4").tobytes()
    assert open(path, "rb").read() == want


def test_round_trip_restores_every_array_and_seen(tmp_path):
    net = network(1)
    path = str(tmp_path / "b.weights")
    save(path, net, seen=42)
    got = blank(net)
    assert load(path, got) == 42
    for a, b in zip(net, got):
        for name in NAMES:
            if getattr(a, name) is not None:
                assert np.array_equal(getattr(a, name), getattr(b, name)), (a.kind, name)


def test_legacy_header_reads_a_32_bit_seen(tmp_path):
    bn = LayerParams("batchnorm", n=3, scales=np.float32([1, 2, 3]), rolling_mean=np.float32([4, 5, 6]),
                     rolling_variance=np.float32([7, 8, 9]))
    path = tmp_path / "old.weights"
    path.write_bytes(struct.pack("<iiii", 0, 1, 0, 77) + np.concatenate(bn.bn_vectors()).astype("<f4").tobytes())
    got = LayerParams("batchnorm", n=3)
    assert load(str(path), [got]) == 77
    assert np.array_equal(got.rolling_variance, [7, 8, 9])


def test_transposed_connected_weights_of_old_files(tmp_path):
    inputs, outputs = 4, 3
    w_out_in = np.arange(outputs * inputs, dtype=np.float32).reshape(outputs, inputs)
    body = np.zeros(outputs, np.float32).tobytes() + w_out_in.T.astype("<f4").tobytes()  # stored inputs x outputs
    path = tmp_path / "t.weights"
    path.write_bytes(struct.pack("<iiii", 0, 1001, 0, 0) + body)
    got = LayerParams("connected", n=outputs, inputs=inputs)
    load(str(path), [got])
    assert np.array_equal(got.weights.reshape(outputs, inputs), w_out_in)


def test_flipped_conv_weights_are_transposed_on_load(tmp_path):
    n, k = 3, 4  # filters, c*size*size
    w = np.arange(n * k, dtype=np.float32).reshape(n, k)
    layer = LayerParams("convolutional", n=n, nweights=n * k, weights=w.T.reshape(-1).copy())
    path = str(tmp_path / "f.weights")
    save(path, [layer])
    got = LayerParams("convolutional", n=n, nweights=n * k, flipped=True)
    load(path, [got])
    assert np.array_equal(got.weights.reshape(n, k), w)


def test_dontsave_dontload_and_dontloadscales(tmp_path):
    net = network(2)
    net[2].dontsave = True
    path = str(tmp_path / "d.weights")
    save(path, net)
    got = blank(net)
    got[1].dontload = True
    load(path, got, cutoff=2)
    assert np.array_equal(got[0].rolling_mean, net[0].rolling_mean)
    assert not got[1].biases.any()
    # dontloadscales: the three BN vectors are not read, so the weights are read from where
    # the file holds the scales (the reference's loader does the same)
    got2 = blank(net)[:1]
    got2[0].dontloadscales = True
    load(path, got2)
    assert not got2[0].scales.any()
    assert np.array_equal(got2[0].weights[:8], net[0].scales)


def test_truncated_file_is_an_error(tmp_path):
    net = network()
    path = tmp_path / "short.weights"
    save(str(path), net)
    path.write_bytes(path.read_bytes()[:-4])
    with pytest.raises(EOFError):
        load(str(path), blank(net))


def test_cpp_host_reads_and_writes_the_same_bytes(tmp_path):
    sys.path.insert(0, os.path.join(os.path.dirname(__file__), "cpp"))
    import build as cpp_build  # tests/cpp/build.py

    exe = cpp_build.build_weights_rt()
    net = network(3)
    src, dst = str(tmp_path / "py.weights"), str(tmp_path / "cpp.weights")
    save(src, net, seen=987654321)
    r = subprocess.run([exe, src, dst], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0, r.stderr
    lines = r.stdout.split("\n")
    assert lines[0] == "seen 987654321"
    for layer, line in zip(net, lines[1:5]):
        if layer.rolling_variance is None:
            assert line == "-"
        else:
            assert np.float32(float(line)) == layer.rolling_variance[0]
    assert open(dst, "rb").read() == open(src, "rb").read()
