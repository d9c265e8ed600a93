"""hilbert_order (src/faster_weathernext/pallas_attn.py:71-82) with the curve codes computed on the GPU.

The 3D Hilbert code of each point (unit-sphere coordinates quantised to `bits` per axis) comes from
the library's CUDA kernel (fwn_hilbert_codes); the permutation is the stable argsort of the codes,
non-finite points last.
"""

import numpy as np
import torch

from faster_weathernext import _lib


def hilbert_codes(lat_deg, lon_deg, bits: int = 10, device=None) -> np.ndarray:
  lat = np.ascontiguousarray(np.asarray(lat_deg, np.float64).ravel())
  lon = np.ascontiguousarray(np.asarray(lon_deg, np.float64).ravel())
  if lat.shape != lon.shape:
    raise ValueError("lat and lon must have the same number of points")
  dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
  la, lo = torch.from_numpy(lat).to(dev), torch.from_numpy(lon).to(dev)
  codes = torch.empty(lat.size, dtype=torch.int64, device=dev)
  _lib.check(_lib.lib().fwn_hilbert_codes(la.data_ptr(), lo.data_ptr(), lat.size, bits, codes.data_ptr(),
                                          torch.cuda.current_stream(dev).cuda_stream))
  return codes.cpu().numpy()


def hilbert_order(lat_deg, lon_deg, bits: int = 10) -> np.ndarray:
  """Permutation sorting points on the sphere along a 3D Hilbert curve (non-finite points last)."""
  return np.argsort(hilbert_codes(lat_deg, lon_deg, bits), kind="stable")
