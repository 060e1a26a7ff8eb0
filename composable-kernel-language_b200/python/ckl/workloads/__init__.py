"""CKL programs whose kernels the sm_100a library implements: the decoder step and the
vector pipeline."""
