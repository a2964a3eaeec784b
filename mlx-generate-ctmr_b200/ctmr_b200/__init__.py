"""B200-native (sm_100a) convolution stack of mlx-generate-ctmr's MAISI networks.

``ops`` exposes the C ABI of ``libctmr_b200.so`` on torch tensors; ``fast_b200``
is the drop-in arithmetic module (the surface of the reference's ``fast_fp32``);
``networks`` holds the VAE decoder, rflow UNet and ControlNet that call it, and
``pipeline`` the samplers and ``run()``.
"""

__version__ = "0.1.0"
