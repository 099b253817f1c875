"""Model families built on b200ar kernels."""
