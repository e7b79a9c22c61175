"""The reference's positional `.weights` format, for the parameters this library trains.

A file is a header (parser.zig:576-579: i32 major = 0, i32 minor = 2, i32 revision = 0,
u64 seen) followed by each layer's parameters in network order, little-endian f32 with no
names or sizes (parser.zig:535-559):

  convolutional  biases[n]; if batch_normalize: scales[n], rolling_mean[n],
                 rolling_variance[n]; weights[nweights]
  connected      biases[outputs]; weights[outputs * inputs]; if batch_normalize: scales,
                 rolling_mean, rolling_variance [outputs]
  batchnorm      scales[c], rolling_mean[c], rolling_variance[c]

Loading (parser.zig:460-530) reads the same order. `seen` is a u64 when
major * 10 + minor >= 2 and both are below 1000, else an i32 (version 0.1 and older); a
major or minor above 1000 marks pre-2015 connected weights stored transposed
(inputs x outputs), which are transposed back on load; a conv layer's `flipped` option
marks weights stored (c/groups*size*size) x n. A layer flagged `dontload` / `dontsave` is
skipped; `dontloadscales` skips a conv / connected layer's three BN vectors on load (the
reference then reads on from where the file holds them, and so does this loader).

This is the round trip of the rolling statistics the fused kernels produce: `pull` copies a
layer's device tensors into its host arrays before `save`, `push` copies loaded arrays back.
The device copies go through torch; the file format itself is plain host code.
"""
from __future__ import annotations

import struct
from dataclasses import dataclass, field

import numpy as np

MAJOR, MINOR, REVISION = 0, 2, 0  # parser.zig:576-578
KINDS = ("convolutional", "connected", "batchnorm")


@dataclass
class LayerParams:
    """One layer's saved parameters (host float32 arrays, filled in place by `load`).

    n: filters (convolutional), outputs (connected) or channels (batchnorm).
    nweights: conv weights (n * c/groups * size * size); for connected, inputs * outputs.
    inputs: connected layers only (for the transposed legacy layout).
    flipped: a conv layer's `flipped` option (weights stored (nweights / n) x n)."""

    kind: str
    n: int
    batch_normalize: bool = False
    nweights: int = 0
    inputs: int = 0
    dontload: bool = False
    dontsave: bool = False
    dontloadscales: bool = False
    flipped: bool = False
    biases: np.ndarray | None = None
    scales: np.ndarray | None = None
    rolling_mean: np.ndarray | None = None
    rolling_variance: np.ndarray | None = None
    weights: np.ndarray | None = None
    device: dict = field(default_factory=dict)  # name -> torch tensor, for pull / push

    def __post_init__(self):
        if self.kind not in KINDS:
            raise ValueError(f"layer kind {self.kind!r} has no parameters in the weights format")
        if self.kind == "connected" and self.nweights == 0:
            self.nweights = self.inputs * self.n
        z = lambda k: np.zeros(k, np.float32)  # noqa: E731
        has_bn = self.kind == "batchnorm" or self.batch_normalize
        if self.kind != "batchnorm":
            self.biases = z(self.n) if self.biases is None else self.biases
            self.weights = z(self.nweights) if self.weights is None else self.weights
        if has_bn:
            self.scales = z(self.n) if self.scales is None else self.scales
            self.rolling_mean = z(self.n) if self.rolling_mean is None else self.rolling_mean
            self.rolling_variance = z(self.n) if self.rolling_variance is None else self.rolling_variance

    def bn_vectors(self):
        return [self.scales, self.rolling_mean, self.rolling_variance]

    def save_order(self):
        """The vectors of this layer in a file, parser.zig:535-559."""
        if self.kind == "convolutional":
            return [self.biases] + (self.bn_vectors() if self.batch_normalize else []) + [self.weights]
        if self.kind == "connected":
            return [self.biases, self.weights] + (self.bn_vectors() if self.batch_normalize else [])
        return self.bn_vectors()

    def pull(self) -> None:
        """Device tensors (self.device[name]) -> host arrays, before a save."""
        for name, t in self.device.items():
            getattr(self, name)[...] = t.detach().reshape(-1).cpu().numpy()

    def push(self) -> None:
        """Host arrays -> device tensors, after a load."""
        import torch

        for name, t in self.device.items():
            t.copy_(torch.from_numpy(getattr(self, name)).reshape(t.shape).to(t.device))


def batchnorm_params(bn, kind: str = "batchnorm", nweights: int = 0) -> LayerParams:
    """LayerParams bound to a `layers.BatchNorm`'s device tensors. kind "convolutional" also
    saves the layer's biases (and `nweights` conv weights, left zero here: the conv GEMM is
    not part of this library); kind "batchnorm" is the standalone layer (scales and rolling
    statistics only)."""
    p = LayerParams(kind=kind, n=bn.filters, batch_normalize=True, nweights=nweights)
    p.device = {"scales": bn.scales, "rolling_mean": bn.rolling_mean, "rolling_variance": bn.rolling_variance}
    if kind != "batchnorm":
        p.device["biases"] = bn.biases
    return p


def save(path: str, layers: list[LayerParams], seen: int = 0) -> None:
    """saveWeights (parser.zig:561-590)."""
    with open(path, "wb") as f:
        f.write(struct.pack("<iiiQ", MAJOR, MINOR, REVISION, seen))
        for layer in layers:
            if layer.dontsave:
                continue
            for a in layer.save_order():
                f.write(np.ascontiguousarray(a, dtype="<f4").tobytes())


def _read_bytes(f, n: int, path: str, what: str) -> bytes:
    buf = f.read(n)
    if len(buf) != n:
        raise EOFError(f"{path}: file ends inside {what} ({len(buf)} of {n} bytes)")
    return buf


def _read(f, a: np.ndarray, path: str) -> None:
    want = a.size * 4
    buf = f.read(want)
    if len(buf) != want:
        raise EOFError(f"{path}: file ends inside a layer's parameters ({len(buf)} of {want} bytes)")
    a[...] = np.frombuffer(buf, dtype="<f4").reshape(a.shape)


def _transpose(a: np.ndarray, rows: int, cols: int) -> None:
    """rows x cols (row-major) -> cols x rows in place, as parser.zig:451-458."""
    a[...] = a.reshape(rows, cols).T.copy().reshape(-1)


def load(path: str, layers: list[LayerParams], start: int = 0, cutoff: int | None = None) -> int:
    """loadWeightsUpto (parser.zig:497-530): fills the layers' arrays in place, returns seen."""
    with open(path, "rb") as f:
        head = f.read(12)
        if len(head) != 12:
            raise EOFError(f"{path}: no weights header")
        major, minor, _revision = struct.unpack("<iii", head)
        if major * 10 + minor >= 2 and major < 1000 and minor < 1000:
            (seen,) = struct.unpack("<Q", _read_bytes(f, 8, path, "the 64-bit seen count"))
        else:
            (seen,) = struct.unpack("<i", _read_bytes(f, 4, path, "the 32-bit seen count"))
            seen = max(0, seen)
        transpose = major > 1000 or minor > 1000
        end = len(layers) if cutoff is None else min(cutoff, len(layers))
        for layer in layers[start:end]:
            if layer.dontload:
                continue
            bn = layer.kind == "batchnorm" or (layer.batch_normalize and not layer.dontloadscales)
            if layer.kind == "convolutional":
                _read(f, layer.biases, path)
                if bn:
                    for a in layer.bn_vectors():
                        _read(f, a, path)
                _read(f, layer.weights, path)
                if layer.flipped:  # parser.zig:468-470
                    _transpose(layer.weights, layer.nweights // layer.n, layer.n)
            elif layer.kind == "connected":
                _read(f, layer.biases, path)
                _read(f, layer.weights, path)
                if transpose:  # stored inputs x outputs
                    _transpose(layer.weights, layer.inputs, layer.n)
                if bn:
                    for a in layer.bn_vectors():
                        _read(f, a, path)
            else:
                for a in layer.bn_vectors():
                    _read(f, a, path)
    return int(seen)
