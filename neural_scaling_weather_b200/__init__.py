"""Blackwell-native (sm_100a) framework for training and running Swin-Transformer
weather emulators on lat-lon grids, with data, tensor and 2-D spatial parallelism."""

__version__ = "0.1.0"
