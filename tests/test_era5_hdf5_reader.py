"""The ERA5 HDF5 reader's indexing, year split, normalisation and invariants, on CPU.

h5py is not installed in this image, so a minimal stand-in for its ``File`` (datasets held as numpy
arrays in ``.npz`` files at the paths the reader expects, indexed with numpy's rules, as h5py's
datasets are for these slices) is put in ``sys.modules`` for the duration of each test.
"""

import os
import sys
import types

import numpy as np
import pytest
import torch

from neural_scaling_weather_b200.data.synthetic import EPOCH0


class _File:
    def __init__(self, path, mode="r"):
        assert mode == "r"
        with open(path, "rb") as f:
            self._d = dict(np.load(f, allow_pickle=False))

    def __getitem__(self, name):
        return self._d[name]

    def __enter__(self):
        return self

    def __exit__(self, *a):
        return False


@pytest.fixture
def fake_h5py(monkeypatch):
    mod = types.ModuleType("h5py")
    mod.File = _File
    monkeypatch.setitem(sys.modules, "h5py", mod)
    return mod


def _save(path, **arrays):
    os.makedirs(os.path.dirname(path), exist_ok=True)
    with open(path, "wb") as f:
        np.savez(f, **arrays)


def _make_store(root, name="era5", years=(2016, 2017), n_t=10, C=3, nlat=9, nlon=16):
    rng = np.random.default_rng(0)
    lat = np.linspace(90, -90, nlat)
    lon = np.arange(nlon) * 360.0 / nlon
    chans = np.array([b"u10m", b"t2m", b"z500"])
    data = {}
    for y in years:
        t0 = (np.datetime64(f"{y}-01-01T00", "h") - EPOCH0).astype(np.int64)
        t = t0 + np.arange(n_t, dtype=np.int64)
        d = rng.standard_normal((n_t, C, nlat, nlon)).astype(np.float32) * 5 + 100
        data[y] = (t, d)
        _save(os.path.join(root, name, f"{y}.h5"), data=d, time=t, channel=chans, latitude=lat, longitude=lon)
    mean = np.array([100.0, 101.0, 99.0], dtype=np.float32)
    std = np.array([5.0, 4.0, 6.0], dtype=np.float32)
    _save(os.path.join(root, name, "stats", "stats_v1.h5"), global_mean=mean, global_std=std)
    inv = rng.random((2, nlat, nlon)).astype(np.float32)
    _save(os.path.join(root, name, "invar", "invariants.h5"), channel=np.array([b"lsm", b"orog"]), data=inv)
    return data, mean, std, inv, lat


def test_hdf5_reader_years_windows_and_normalisation(tmp_path, fake_h5py):
    from neural_scaling_weather_b200.data.era5hdf5 import Era5HDF5Dataset

    data, mean, std, inv, lat = _make_store(str(tmp_path))
    # training on both years: a window that crosses the year boundary reads from both files
    ds = Era5HDF5Dataset(root=str(tmp_path), name="era5", tag="v1", mode="train", dt_scale=2,
                         num_rollout_steps=1, invariants=["lsm", "orog", "coslat"])
    assert ds.years == [2016, 2017] and ds.era5_channels == ["u10m", "t2m", "z500"]
    assert ds.n_samples_total == 20 - 2 and ds.nlat == 8  # south-pole row dropped
    x = ds.generate(ds.window_hours(9))  # hours 9 of 2016 and 1 of 2017
    assert x.shape == (2, 3, 8, 16)
    want = np.stack([data[2016][1][9], data[2017][1][1]])[:, :, :-1]
    want = (want - mean[None, :, None, None]) / std[None, :, None, None]
    assert torch.allclose(x, torch.from_numpy(want), atol=1e-6)
    # invariants: lsm as stored, orog min-max normalised, coslat computed; pole row dropped
    assert ds.invar.shape == (3, 8, 16)
    assert np.allclose(ds.invar[0], inv[0, :-1])
    o = inv[1, :-1]
    assert np.allclose(ds.invar[1], (o - o.min()) / o.max())
    assert np.allclose(ds.invar[2], np.cos(np.deg2rad(lat[:-1]))[:, None] * np.ones((1, 16)))


def test_hdf5_reader_holds_out_validation_and_test_years(tmp_path, fake_h5py):
    from neural_scaling_weather_b200.data.era5hdf5 import Era5HDF5Dataset

    data, mean, std, _, _ = _make_store(str(tmp_path), years=(2016, 2017, 2018))
    kw = dict(root=str(tmp_path), name="era5", tag="v1", valid_years=[2017], test_years=[2018])
    assert Era5HDF5Dataset(mode="train", **kw).years == [2016]
    val = Era5HDF5Dataset(mode="valid", **kw)
    assert val.years == [2017] and val.n_samples_total == 10 - 1  # two-step windows
    x = val.generate(val.window_hours(3))
    want = (data[2017][1][3:5, :, :-1] - mean[None, :, None, None]) / std[None, :, None, None]
    assert torch.allclose(x, torch.from_numpy(want), atol=1e-6)
    assert Era5HDF5Dataset(mode="test", **kw).years == [2018]


def test_hdf5_reader_reports_missing_h5py(tmp_path, monkeypatch):
    from neural_scaling_weather_b200.data import era5hdf5

    monkeypatch.setitem(sys.modules, "h5py", None)  # import fails
    with pytest.raises(RuntimeError, match="h5py"):
        era5hdf5.Era5HDF5Dataset(root=str(tmp_path), name="none")
