"""maloq_b200 subpackage."""
