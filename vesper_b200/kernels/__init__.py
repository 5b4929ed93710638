"""The fused kernels of the column hot path, behind the reference's ``vesper.kernels`` names."""
