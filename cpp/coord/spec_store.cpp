#include "spec_store.h"

#include <unistd.h>

#include <cctype>
#include <cstdio>

#include "util.h"

namespace es {

namespace {

class FileSpecStore : public SpecStore {
 public:
  explicit FileSpecStore(std::string dir) : dir_(std::move(dir)) {}
  bool put(const std::string& key, const std::string& bytes) override {
    const std::string path = dir_ + "/" + key;
    mkdirs(path.substr(0, path.rfind('/')));
    return write_file_atomic(path, bytes);
  }
  bool remove(const std::string& key) override { return ::unlink((dir_ + "/" + key).c_str()) == 0; }
  bool list(const std::string& prefix, std::map<std::string, std::string>& out) override {
    const auto slash = prefix.rfind('/');
    const std::string sub = slash == std::string::npos ? "" : prefix.substr(0, slash + 1);
    for (auto& f : list_dir(dir_ + "/" + sub)) {
      const std::string key = sub + f;
      if (key.compare(0, prefix.size(), prefix) != 0 || f.find(".tmp") != std::string::npos) continue;
      std::string data;
      if (read_file(dir_ + "/" + key, data)) out[key] = data;
    }
    return true;
  }
  std::string where() const override { return dir_; }

 private:
  std::string dir_;
};

class KubeSpecStore : public SpecStore {
 public:
  KubeSpecStore(KubeClient k, std::string ns) : k_(std::move(k)), ns_(std::move(ns)) {}
  std::string coll() const { return "/apis/everserve.ai/v1/namespaces/" + ns_ + "/everservestates"; }

  bool put(const std::string& key, const std::string& bytes) override {
    const std::string name = object_name_of(key);
    for (int attempt = 0; attempt < 5; attempt++) {
      std::string out, rv;
      const int g = k_.request("GET", coll() + "/" + name, "", out);
      Json j;
      if (g == 200 && Json::parse(out, j))
        if (const Json* m = j.get("metadata"))
          if (const Json* r = m->get("resourceVersion")) rv = r->str;
      const std::string obj = "{\"apiVersion\":\"everserve.ai/v1\",\"kind\":\"EverserveState\",\"metadata\":{\"name\":\"" +
                              name + "\",\"namespace\":\"" + json_escape(ns_) + "\"" +
                              (rv.empty() ? "" : ",\"resourceVersion\":\"" + json_escape(rv) + "\"") +
                              "},\"spec\":{\"key\":\"" + json_escape(key) + "\",\"data\":\"" + base64_encode(bytes) + "\"}}";
      const int w = g == 404 ? k_.request("POST", coll(), obj, out) : k_.request("PUT", coll() + "/" + name, obj, out);
      if (w == 200 || w == 201) return true;
      if (w != 409) {
        ES_WARN("spec store %s: writing %s answered %d", ns_.c_str(), key.c_str(), w);
        return false;
      }
    }
    return false;
  }

  bool remove(const std::string& key) override {
    std::string out;
    const int d = k_.request("DELETE", coll() + "/" + object_name_of(key), "", out);
    return d == 200 || d == 202 || d == 404;
  }

  bool list(const std::string& prefix, std::map<std::string, std::string>& out) override {
    std::string body;
    if (k_.request("GET", coll(), "", body, 10000) != 200) return false;
    Json j;
    if (!Json::parse(body, j)) return false;
    if (const Json* items = j.get("items"))
      for (auto& it : items->arr) {
        const Json* spec = it.get("spec");
        const Json* key = spec ? spec->get("key") : nullptr;
        const Json* data = spec ? spec->get("data") : nullptr;
        if (!key || key->str.compare(0, prefix.size(), prefix) != 0) continue;
        std::string bytes;
        if (data && base64_decode(data->str, bytes)) out[key->str] = bytes;
      }
    return true;
  }
  std::string where() const override { return "k8s:" + ns_; }

 private:
  KubeClient k_;
  std::string ns_;
};

}  // namespace

std::string object_name_of(const std::string& key) {
  std::string n;
  for (char c : key) {
    const char l = (char)std::tolower((unsigned char)c);
    n.push_back((l >= 'a' && l <= 'z') || (l >= '0' && l <= '9') ? l : '-');
  }
  while (!n.empty() && n.front() == '-') n.erase(n.begin());
  if (n.size() > 40) n.resize(40);
  uint32_t h = 2166136261u;  // FNV-1a of the key: two keys that read alike stay apart
  for (char c : key) h = (h ^ (uint8_t)c) * 16777619u;
  char suf[16];
  std::snprintf(suf, sizeof suf, "-%08x", h);
  return "es-" + n + suf;
}

std::unique_ptr<SpecStore> make_spec_store(const std::string& spec) {
  if (spec.empty()) return nullptr;
  if (spec.rfind("k8s:", 0) == 0) return std::make_unique<KubeSpecStore>(KubeClient::from_env(), spec.substr(4));
  return std::make_unique<FileSpecStore>(spec);
}

}  // namespace es
