#!/bin/sh
# Builds quail_b200/_native*.so alone (the host runtime, no CUDA); setup.py builds it too.
set -e
cd "$(dirname "$0")/../.."
PYINC=$(python -c "import sysconfig;print(sysconfig.get_paths()['include'])")
PBINC=$(python -c "import pybind11;print(pybind11.get_include())")
EXT=$(python -c "import sysconfig;print(sysconfig.get_config_var('EXT_SUFFIX'))")
g++ -O3 -std=c++20 -fPIC -shared -fvisibility=hidden -I"$PYINC" -I"$PBINC" quail_b200/native/*.cpp -lpthread -o "quail_b200/_native$EXT"
