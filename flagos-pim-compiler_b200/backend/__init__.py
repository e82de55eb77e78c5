"""B200 HAL package.  ``backend.hal_cuda.CudaBackend`` is the drop-in for the
reference's ``backend.hal_numpy.NumpyBackend``; the C-ABI binding lives in
``backend._native`` and the plan lowering in ``backend.cuda_kernels`` /
``backend.cuda_collectives``."""
