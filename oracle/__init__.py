"""CPU oracle for the GDN layer: test infrastructure, never imported by the product library."""
