"""NumPy-backed stand-in for the ``mlx`` package (see ``mlx.core``)."""
