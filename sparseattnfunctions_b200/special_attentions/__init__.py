"""Drop-in mirror of the reference special_attentions package (sm_100a kernels inside)."""
