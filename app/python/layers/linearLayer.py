"""Drop-in name for the reference's app/python/layers/linearLayer.py."""
from directaccesskernel_b200.layers import Linear, LinearHorizontal  # noqa: F401
