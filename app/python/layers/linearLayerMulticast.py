"""Drop-in name for the reference's app/python/layers/linearLayerMulticast.py."""
from directaccesskernel_b200.layers import LinearHorizontalMulticast, LinearMulticast  # noqa: F401
