"""Algorithm cases.  Only ``rbf`` (the Gaussian RBF kernel matrix) is built here."""
