"""Sinkhorn attention operators backed by libdfsink.so."""
