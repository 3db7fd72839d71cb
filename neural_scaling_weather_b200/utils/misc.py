"""Grid helpers and test fixtures (``utils/misc_utils.py:14-78`` of the reference)."""

from __future__ import annotations

import numpy as np
import torch

from ..parallel import comm


def get_spatial_coords(locations):
    """(lat[deg], lon[deg]) -> unit-sphere xyz of the mesh, shape (nlat, nlon, 3)."""
    lat, lon = torch.as_tensor(np.asarray(locations[0])), torch.as_tensor(np.asarray(locations[1]))
    lat, lon = torch.meshgrid(lat, lon, indexing="ij")
    lat, lon = torch.deg2rad(lat), torch.deg2rad(lon)
    return torch.stack((torch.cos(lat) * torch.cos(lon), torch.cos(lat) * torch.sin(lon),
                        torch.sin(lat)), dim=-1)


def get_local_slice(sizes, rank):
    start = sum(sizes[:rank])
    return slice(start, start + sizes[rank])


def build_spherical_area_weights(latitudes):
    """cos(lat) normalised to mean 1, shape (nlat,)."""
    c = np.cos(np.deg2rad(np.asarray(latitudes, dtype=np.float64)))
    return torch.from_numpy(c / c.mean())


def create_dummy_metadata(H, W, C):
    return {
        "area_weights": torch.rand(H, W, dtype=torch.float32),
        "coords": torch.rand(H, W, 3, dtype=torch.float32),
        "sp_shapes": [[H], [W]],
        "sp_slices": [[slice(0, H)], [slice(0, W)]],
        "channels": [f"ch{i}" for i in range(C)],
        "n_channels": C,
        "spatial_dims": [H, W],
    }


def split_dummy_metadata(metadata, sp1_shapes, sp2_shapes):
    s1 = get_local_slice(sp1_shapes, comm.get_rank("sp1"))
    s2 = get_local_slice(sp2_shapes, comm.get_rank("sp2"))
    return {
        "area_weights": metadata["area_weights"][s1, s2],
        "coords": metadata["coords"][s1, s2, :],
        "sp_shapes": [sp1_shapes, sp2_shapes],
        "sp_slices": [s1, s2],
        "channels": metadata["channels"],
        "n_channels": metadata["n_channels"],
        "spatial_dims": [sp1_shapes[comm.get_rank("sp1")], sp2_shapes[comm.get_rank("sp2")]],
    }
