"""cliffordcuda_b200: B200 (sm_100a) kernels for Cl(p, q, r) multivector
products, product layers and rotors, behind the CliffordCUDA API."""
from .algebra import CliffordAlgebra
from .products import (geom_prod, wedge_prod, inner_prod, left_contract, right_contract,
                       regressive_prod)
from .layers import (GeometricProductLayer, WedgeProductLayer, InnerProductLayer,
                     LeftContractionLayer, RightContractionLayer, RegressiveProductLayer,
                     RotorLayer)


def reverse(x):
    """Reversion of (batch, 2^n) multivectors: grade k -> (-1)^(k(k-1)/2)."""
    import torch
    dim = x.shape[-1]
    idx = torch.arange(dim, device=x.device)
    k = torch.zeros(dim, device=x.device, dtype=torch.long)
    for t in range(dim.bit_length() - 1):
        k += (idx >> t) & 1
    return x * torch.where(((k * (k - 1) // 2) % 2) == 1, -1.0, 1.0).to(x.dtype)


__all__ = [
    "CliffordAlgebra",
    "geom_prod", "wedge_prod", "inner_prod", "left_contract", "right_contract",
    "regressive_prod", "reverse",
    "GeometricProductLayer", "WedgeProductLayer", "InnerProductLayer",
    "LeftContractionLayer", "RightContractionLayer", "RegressiveProductLayer",
    "RotorLayer",
]
__version__ = "0.1.0"
