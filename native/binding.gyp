{
  "targets": [
    {
      "target_name": "tabby_napi",
      "sources": ["tabby_napi.c"],
      "include_dirs": ["../include"],
      "libraries": ["-L<(module_root_dir)/../tabby_b200/lib", "-ltabbysample",
                    "-Wl,-rpath,<(module_root_dir)/../tabby_b200/lib"]
    }
  ]
}
