"""ORACLE -- test infrastructure only (see reference_model.py). The product
package never imports this directory."""
