"""CPU oracle of the VoxCPM2 patch loop -- test infrastructure only.

Used by tests/, __graft_entry__.smoke() and bench.py's CPU baseline as the
checker. The product (voxcpm2_b200 / libvoxcpm2_cuda.so) never imports it.
"""
from .oracle import *  # noqa: F401,F403
