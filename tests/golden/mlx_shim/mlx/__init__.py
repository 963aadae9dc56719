"""NumPy-backed stand-in for the ``mlx`` package (fixture generation only).

Lets ``make_golden.py`` import the reference's pure-Python CPU path
(``mlx_foveated.py``, ``turbo_quantize.py``, ``turbo_constants.py``) in a
container without MLX.  Arrays are plain ``numpy.ndarray``.
"""
