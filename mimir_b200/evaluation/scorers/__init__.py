"""Sample scorers."""
