"""cliffordcuda_b200: B200 (sm_100a) kernels for Cl(p, q, r) multivector
products, product layers and rotors, behind the CliffordCUDA API."""
from .algebra import CliffordAlgebra
from .products import (geom_prod, wedge_prod, inner_prod, left_contract, right_contract,
                       regressive_prod)
from .layers import (GeometricProductLayer, WedgeProductLayer, InnerProductLayer,
                     LeftContractionLayer, RightContractionLayer, RegressiveProductLayer,
                     RotorLayer)
from .blade_maps import reverse


__all__ = [
    "CliffordAlgebra",
    "geom_prod", "wedge_prod", "inner_prod", "left_contract", "right_contract",
    "regressive_prod", "reverse",
    "GeometricProductLayer", "WedgeProductLayer", "InnerProductLayer",
    "LeftContractionLayer", "RightContractionLayer", "RegressiveProductLayer",
    "RotorLayer",
]
__version__ = "0.1.0"
