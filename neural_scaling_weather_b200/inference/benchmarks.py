"""Third-party forecasts scored in place of the model (``inference.run_benchmark``).

The reference can score GraphCast or ECMWF HRES forecasts from WeatherBench2 against the same
targets, leads and metrics as its own model (``utils/inferencer.py:201-285``): the forecast of each
initial condition is read for every lead, its variables are matched to the model's channels by
name, the latitude axis (stored south to north on 721 rows) is flipped to the model's north-to-south
order and the south-pole row is dropped, and the result is scored in physical units.

Here a :class:`ForecastSource` supplies the forecast fields and :func:`assemble` builds this rank's
(lead, channel, lat, lon) shard from them.  :class:`ZarrForecast` reads a WeatherBench2-layout zarr
store with xarray (the named WeatherBench2 stores live on Google Cloud Storage: they need network
access and the ``xarray`` / ``zarr`` / ``gcsfs`` packages); any other source with the same
``fetch`` method can be handed to the inferencer instead (``Inferencer.bench_source``).
"""

from __future__ import annotations

from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np
import torch

# model variable -> WeatherBench2 variable name (the external dataset's naming; channels whose
# variable is not listed, or that a store lacks, are left at zero as the reference does)
WB2_NAMES: Dict[str, str] = {
    "u10m": "10m_u_component_of_wind",
    "v10m": "10m_v_component_of_wind",
    "t2m": "2m_temperature",
    "msl": "mean_sea_level_pressure",
    "z": "geopotential",
    "q": "specific_humidity",
    "t": "temperature",
    "u": "u_component_of_wind",
    "v": "v_component_of_wind",
}

# the public WeatherBench2 stores the reference names
WB2_STORES: Dict[str, str] = {
    "graphcast": "gs://weatherbench2/datasets/graphcast/2020/date_range_2019-11-16_2021-02-01_12_hours.zarr",
    "hres": "gs://weatherbench2/datasets/hres/2016-2022-0012-1440x721.zarr",
}


def split_channel(name) -> Tuple[str, Optional[int]]:
    """``"z500"`` -> ``("z", 500)``; ``"t2m"`` / ``"u10m"`` (surface names ending in a letter) -> (name, None)."""
    if isinstance(name, bytes):
        name = name.decode("utf-8")
    stem = name.rstrip("0123456789")
    if stem != name and len(name) > 1:
        return stem, int(name[len(stem):])
    return name, None


class ForecastSource:
    """A third-party forecast: ``fetch(ic, leads_h, var, level)`` returns an array (n_leads, n_lat, n_lon)
    on the source's own grid (latitudes south to north, 721 rows for 0.25 degree) or None when the
    source has no such variable / level."""

    def fetch(self, ic: np.datetime64, leads_h: Sequence[int], var: str, level: Optional[int]):
        raise NotImplementedError


class ZarrForecast(ForecastSource):
    """A WeatherBench2-layout zarr store (dims time, prediction_timedelta, [level,] latitude, longitude)."""

    def __init__(self, path: str):
        try:
            import xarray as xr
        except ImportError as e:
            raise RuntimeError("scoring a WeatherBench2 forecast needs xarray and zarr (and gcsfs for gs:// "
                               "stores), which are not installed") from e
        self.path = path
        self.ds = xr.open_zarr(path)
        self._ic = None
        self._sel = None

    def fetch(self, ic, leads_h, var, level):
        key = (ic, tuple(leads_h))
        if self._ic != key:
            self._sel = self.ds.sel(time=ic, prediction_timedelta=[np.timedelta64(int(h), "h") for h in leads_h])
            self._ic = key
        wb = WB2_NAMES.get(var)
        if wb is None or wb not in self._sel.data_vars:
            return None
        arr = self._sel[wb]
        if level is not None:
            if "level" not in arr.dims or level not in arr["level"].values:
                return None
            arr = arr.sel(level=level)
        elif "level" in arr.dims:
            return None
        return np.asarray(arr.values, dtype=np.float32)


def make_source(inf_cfg) -> ForecastSource:
    """The source ``inference.run_benchmark`` names: ``graphcast`` / ``hres`` (``inference.benchmark_path``
    overrides the store's location, e.g. a local copy)."""
    name = str(inf_cfg.run_benchmark)
    if name not in WB2_STORES:
        raise ValueError(f"invalid benchmark {name!r}: expected one of {sorted(WB2_STORES)}")
    path = inf_cfg.get("benchmark_path", None) or WB2_STORES[name]
    return ZarrForecast(path)


def assemble(source: ForecastSource, ic, leads_h: Sequence[int], channels: Sequence, lat_slice: slice,
             lon_slice: slice, n_lat: int) -> Tuple[torch.Tensor, List[int]]:
    """This rank's shard (n_leads, C, H_l, W_l) fp32 of the forecast in physical units, on the model's grid:
    latitudes flipped to north-to-south and cut to the model's ``n_lat`` rows (the south pole row of a
    721-row grid is dropped).  Also returns the channel indices the source supplied."""
    n = len(leads_h)
    rows = lat_slice.stop - lat_slice.start
    cols = lon_slice.stop - lon_slice.start
    out = torch.zeros(n, len(channels), rows, cols, dtype=torch.float32)
    found = []
    for ci, ch in enumerate(channels):
        var, level = split_channel(ch)
        a = source.fetch(ic, leads_h, var, level)
        if a is None:
            continue
        a = np.asarray(a, dtype=np.float32)
        if a.ndim != 3 or a.shape[0] != n:
            raise ValueError(f"benchmark field {ch}: expected ({n}, lat, lon), got {a.shape}")
        a = a[:, ::-1][:, :n_lat]  # north to south, pole row dropped
        out[:, ci] = torch.from_numpy(np.ascontiguousarray(a[:, lat_slice, lon_slice]))
        found.append(ci)
    return out, found
