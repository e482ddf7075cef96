"""torch-helion on B200: the torch-helion front end with sm_100a kernels."""
