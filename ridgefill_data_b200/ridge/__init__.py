"""Closed-form ridge maps: sufficient statistics, fits (eigen and Cholesky), map files, the fit driver."""
