{
  "targets": [
    {
      "target_name": "bgtq",
      "sources": ["bgtq_napi.c"],
      "include_dirs": ["../../include"],
      "libraries": ["-L<(module_root_dir)/../bgtq", "-lbgtq", "-Wl,-rpath,<(module_root_dir)/../bgtq"],
      "cflags": ["-std=c11", "-O2", "-Wall"]
    }
  ]
}
